"""Generate the golden fixtures under tests/golden/ from the reference itself.

Runs the reference engine's own CPU path (oracle/_ref/libxlref.so, compiled
from the reference sources by oracle/Makefile) on seeded inputs and stores
its outputs.  The inputs are not stored: every case regenerates them from a
numpy seed (see case_inputs), so the fixtures stay small.  The tests in
tests/test_oracle_pin.py check the oracle port against these files.

    CUDA_VISIBLE_DEVICES= python tests/golden/make_golden.py [--full]

--full also pins the XingLing-0.68B shape (writes the 2.75 GB seeded weight
tree to $XL_WEIGHT_CACHE/full first).
"""
import os
import sys

os.environ["CUDA_VISIBLE_DEVICES"] = ""
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "xingling-cpp_b200"), os.path.dirname(HERE)]

import numpy as np  # noqa: E402

import oracle as O  # noqa: E402
import xl_synth as S  # noqa: E402
from golden_cases import OP_CASES, SAMPLER_CASES, case_inputs, sampler_logits  # noqa: E402

WEIGHT_CACHE = os.environ.get("XL_WEIGHT_CACHE", "/tmp/xl_weights")


def ops() -> dict:
    out = {}
    for name in OP_CASES:
        a = case_inputs(name)
        kind = OP_CASES[name]["kind"]
        if kind == "linear":
            out[name] = O.ref_linear(a["x"], a["w"], a["b"])
        elif kind == "linear_vec":
            out[name] = O.ref_linear(a["x"], a["w"], a["b"], vec=True)
        elif kind == "rmsnorm":
            out[name] = O.ref_rmsnorm(a["x"], a["gamma"])
        elif kind == "rope":
            out[name] = O.ref_rope(a["x"], None)
        elif kind == "rope_vec":
            out[name] = O.ref_rope(a["x"], OP_CASES[name]["pos"])
        elif kind == "attn_prefill":
            o, kc, vc = O.ref_attn_prefill(a["q"], a["k"], a["v"], OP_CASES[name]["max_ctx"])
            n = a["q"].shape[0]
            out[name], out[name + ".kc"], out[name + ".vc"] = o, kc[:n], vc[:n]
        elif kind == "attn_decode":
            pos = OP_CASES[name]["pos"]
            o, kc, vc = O.ref_attn_decode(a["q"], a["k"], a["v"], a["kc"], a["vc"], pos)
            out[name], out[name + ".kc"], out[name + ".vc"] = o, kc[: pos + 1], vc[: pos + 1]
        elif kind == "embedding":
            rows, logits = O.ref_embedding(a["table"], a["ids"], a["h"])
            out[name + ".rows"], out[name] = rows, logits
        elif kind == "swiglu":
            out[name] = O.ref_swiglu(a["x"], a["w1"], a["b1"], a["v"], a["bv"], a["w2"], a["b2"])
        else:
            raise ValueError(kind)
    return out


def sampler() -> dict:
    out = {}
    for name, c in SAMPLER_CASES.items():
        tok, r = O.ref_sample(sampler_logits(c), c["T"], c["p"], c["rp"], c["rep"], c["mt_seed"])
        out[name + ".token"] = np.array([tok], np.int64)
        out[name + ".r"] = np.array([r], np.float32)
    return out


def model(shape: S.ModelShape, tag: str, n_prompt: int, prompt_seed: int, steps: int, full_logits: bool) -> dict:
    wdir = S.write_weight_tree(os.path.join(WEIGHT_CACHE, tag), shape)
    ref = O.Ref(shape)
    ref.load(wdir)
    ids = S.prompt_ids(prompt_seed, n_prompt, shape.vocab)
    out = {"ids": np.array(ids, np.int64)}
    logits = ref.prefill(ids)
    toks = []
    for step in range(steps + 1):
        key = f"step{step}"
        if full_logits:
            out[key] = logits
        else:
            top = np.argsort(-logits, kind="stable")[:64]
            out[key + ".top_ids"] = top.astype(np.int64)
            out[key + ".top_vals"] = logits[top]
            out[key + ".stride"] = logits[::97].copy()
            out[key + ".stats"] = np.array([logits.min(), logits.max(), logits.astype(np.float64).sum(),
                                            (logits.astype(np.float64) ** 2).sum()])
        tok = int(np.argmax(logits))
        toks.append(tok)
        if step < steps:
            logits = ref.decode(tok)
    out["greedy"] = np.array(toks, np.int64)
    out["kv_n"] = np.array([ref.kv_n(l) for l in range(shape.layers)], np.int64)
    k, v = ref.kv(shape.layers - 1, n_prompt + steps)
    out["kv_last.k_sum"] = np.array([k.astype(np.float64).sum(), np.abs(k).astype(np.float64).sum()])
    out["kv_last.v_sum"] = np.array([v.astype(np.float64).sum(), np.abs(v).astype(np.float64).sum()])
    return out


def main() -> None:
    O.build(ref=True)
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **ops())
    np.savez_compressed(os.path.join(HERE, "sampler.npz"), **sampler())
    np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), **model(S.TINY, "tiny", 17, 0, 4, True))
    if "--full" in sys.argv:
        np.savez_compressed(os.path.join(HERE, "full_model.npz"), **model(S.FULL, "full", 32, 0, 8, False))
    print("golden fixtures written to", HERE)
    sys.stdout.flush()
    os._exit(0)  # skip the reference's Embedding destructor (it exits on GPU-less hosts)


if __name__ == "__main__":
    main()
