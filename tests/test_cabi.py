"""CPU checks of the drop-in boundary: libxl_engine.so loads and exports every
function include/xl_engine.h declares; the llm_cpp_engine module mirrors the
reference's pybind11 surface (src/bindings.cpp:7-39); host-only helpers
(Philox stream, TP shard plan) behave.  No compute call needs a GPU here."""
import ctypes as C
import inspect

import numpy as np
import pytest

import xl_capi as X
import xl_synth as S


def test_library_exports_every_declared_symbol(built):
    lib = C.CDLL(X.LIB_PATH)
    declared = X.declared_functions()
    assert len(declared) >= 30
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing


def test_config_default_matches_reference_constants(built):
    lib = C.CDLL(X.LIB_PATH)

    class Cfg(C.Structure):
        _fields_ = [(n, C.c_int) for n in ("layers", "hidden", "heads", "ffn", "vocab", "max_ctx")] + \
                   [("rope_base", C.c_float)]

    cfg = Cfg()
    lib.xl_config_default(C.byref(cfg))
    # src/inference.cu:19-28
    assert (cfg.layers, cfg.hidden, cfg.heads, cfg.ffn, cfg.vocab, cfg.max_ctx) == (16, 1536, 24, 4096, 151669, 768)
    assert cfg.rope_base == 10000.0


def test_philox_stream_matches_host_generator(built):
    lib = C.CDLL(X.LIB_PATH)
    lib.xl_philox_uniforms.argtypes = [C.c_uint64, C.c_uint64, C.c_int, C.c_void_p]
    out = np.empty(1000, np.float32)
    assert lib.xl_philox_uniforms(3, 17, 1000, out.ctypes.data) == 0
    assert np.array_equal(out, S.philox_uniforms(3, 1000, start=17))
    # Random123 known-answer vector: philox4x32-10, counter 0, key 0 -> x0 = 0x6627e8d5
    assert int(S.philox4x32_10(np.array([0], np.uint64), 0)[0]) == 0x6627E8D5
    assert np.all((out >= 0) & (out < 1))


def _plan(lib, tp, rank, vocab=151669, heads=24, ffn=4096):
    class Cfg(C.Structure):
        _fields_ = [(n, C.c_int) for n in ("layers", "hidden", "heads", "ffn", "vocab", "max_ctx")] + \
                   [("rope_base", C.c_float)]

    cfg = Cfg(16, heads * 64, heads, ffn, vocab, 768, 10000.0)
    out = (C.c_int * 5)()
    rc = lib.xl_tp_plan(C.byref(cfg), tp, rank, out)
    return rc, list(out)


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_tp_plan_partitions(built, tp):
    lib = C.CDLL(X.LIB_PATH)
    plans = [_plan(lib, tp, r) for r in range(tp)]
    assert all(rc == 0 for rc, _ in plans)
    assert sum(p[0] for _, p in plans) == 24 and all(p[1] == p[0] * 64 for _, p in plans)
    assert sum(p[2] for _, p in plans) == 4096
    # contiguous vocab shards covering [0, 151669) exactly
    begin = 0
    for _, p in plans:
        assert p[3] == begin
        begin += p[4]
    assert begin == 151669
    assert {p[0] for _, p in plans} == {24 // tp}


def test_tp_plan_rejects_bad_splits(built):
    lib = C.CDLL(X.LIB_PATH)
    assert _plan(lib, 5, 0)[0] != 0  # 5 does not divide 24 heads
    assert _plan(lib, 2, 2)[0] != 0  # rank out of range
    assert _plan(lib, 0, 0)[0] != 0


def test_module_surface_mirrors_reference(built):
    import llm_cpp_engine as m

    cls = m.InferenceEngine
    for name in ("load", "to", "device", "next_token", "im_start_id", "im_end_id", "nl_id", "role_id_user",
                 "role_id_assistant"):
        assert hasattr(cls, name), name
    doc = cls.next_token.__doc__
    # overload order (list before int) and keyword defaults of src/bindings.cpp:15-33
    assert doc.index("1. next_token(self: llm_cpp_engine.InferenceEngine, input_ids") < \
        doc.index("2. next_token(self: llm_cpp_engine.InferenceEngine, token")
    for kw, val in (("temperature", 0.7), ("top_p", 0.9), ("repetition_penalty", 1.1)):
        shown = f"{float(np.float32(val))!r}"[:8]
        assert doc.count(kw) == 2 and doc.count(f"= {shown}") >= 2, (kw, shown)
    with pytest.raises(ValueError):
        m.InferenceEngine("cpu")  # no CPU fallback in the product
    with pytest.raises(ValueError):
        m.InferenceEngine("tpu")


def test_module_reports_missing_gpu_as_error(built):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import llm_cpp_engine as m

    with pytest.raises(RuntimeError):
        m.InferenceEngine("cuda")


def test_kernel_launch_counter(built):
    import ctypes as C

    import llm_cpp_engine as m

    lib = C.CDLL(X.LIB_PATH)
    lib.xl_kernel_launches.restype = C.c_longlong
    n = lib.xl_kernel_launches()
    assert n >= 0 and m.kernel_launches() >= 0
    # launches are only counted by launchers: nothing ran here, so nothing changed
    assert lib.xl_kernel_launches() == n


def test_weight_tree_is_deterministic(tmp_path):
    sh = S.ModelShape(layers=1, hidden=64, heads=1, ffn=64, vocab=100, max_ctx=16)
    a = S.write_weight_tree(str(tmp_path / "a"), sh)
    b = S.write_weight_tree(str(tmp_path / "b"), sh)
    for rel, shape, kind in S.weight_specs(sh):
        x = np.fromfile(f"{a}/{rel}", np.float32)
        y = np.fromfile(f"{b}/{rel}", np.float32)
        assert x.size == int(np.prod(shape)) and np.array_equal(x, y)
        if kind == "ones":
            assert np.all(x == 1.0)
        else:
            assert abs(float(x.std()) - 0.02) < 0.01
    assert sh.weight_bytes() == sum(4 * int(np.prod(s)) for _, s, _ in S.weight_specs(sh))
    assert S.FULL.weight_bytes() == 2_745_012_224  # embedding + 16 layers + final norm, fp32


def test_bench_byte_model_matches_survey():
    import bench

    # 2,745,018,368 + 196,608 * ctx bytes per decode token
    b0 = bench.decode_bytes_per_token(S.FULL, 0)
    b1 = bench.decode_bytes_per_token(S.FULL, 1)
    assert int(b0) == 2_745_018_368  # all weights + the gathered embedding row
    assert int(b1 - b0) == 196_608
    assert abs(bench.prefill_flops(S.FULL, 512) / 1e9 - 477.2) < 0.5
    assert inspect.isfunction(bench.reference_arm)
