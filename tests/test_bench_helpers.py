"""Host-side helpers of bench.py (no GPU): the phase-timeline summary of the
persistent kernel's own %globaltimer stamps, and the roofline denominators."""
import importlib.util
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("xl_bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_phase_summary_of_a_synthetic_timeline():
    b = _bench()
    sms, layers = 148, 16
    a = np.zeros((sms, 5 * layers + 1, 5), dtype=np.uint64)
    t = 10_000_000
    for ph in range(5 * layers + 1):
        kind = 5 if ph == 5 * layers else ph % 5
        stage, cons = 1000 * (kind + 1), 2000 * (kind + 1)
        a[:, ph, 0] = t
        a[:, ph, 1] = t + stage
        a[:, ph, 2] = t + stage + cons
        if kind == 1:
            a[1:, ph, 0] = 0  # CTAs without an attention item stamp only the end
            a[1:, ph, 1] = 0
        t += stage + cons
    r = b.phase_summary(a.tobytes(), sms, layers)
    for kind, name in enumerate(b.PHASE_KINDS + ["LM head"]):
        assert r[name]["staging_us"] == (kind + 1) * 1.0
        assert r[name]["consume_us"] == (kind + 1) * 2.0
        assert r[name]["phase_us"] == (kind + 1) * 3.0
    assert r["step_us"] == (t - 10_000_000) / 1e3


def test_peaks_fall_back_without_the_measured_file(tmp_path, monkeypatch):
    b = _bench()
    monkeypatch.setattr(b, "ROOT", str(tmp_path))
    pk, kind = b.peaks()
    assert kind == "fallback" and pk["hbm_gbs"] > 0 and pk["bf16_tflops"] > 0


def test_library_record_names_the_timed_library(tmp_path, monkeypatch):
    """The reference arm reports which library it timed: its path relative to
    the repository, its size and hash, and whether the process maps it."""
    b = _bench()
    lib = tmp_path / "libfake.so"
    lib.write_bytes(b"\x7fELF" + b"\0" * 60)
    monkeypatch.setattr(b, "ROOT", str(tmp_path))
    rec = b.library_record(str(lib))
    assert rec["path"] == "libfake.so" and rec["bytes"] == 64 and len(rec["sha256_16"]) == 16
    assert rec["mapped"] is False  # not loaded by this process
    assert "restatement" in rec["what"]


def test_engine_options_from_the_command_line(monkeypatch):
    b = _bench()
    seen = []

    class Eng:
        def set_option(self, k, v):
            seen.append((k, v))

    monkeypatch.setattr(b, "ENGINE_OPTS", {"tag_split": 1, "tp_merge": 0})
    e = Eng()
    assert b.apply_opts(e) is e
    assert seen == [("tag_split", 1), ("tp_merge", 0)]
