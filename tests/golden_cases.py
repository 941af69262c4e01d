"""Seeded inputs of the golden cases (shared by tests/golden/make_golden.py and
the tests).  Shapes and scales follow the reference's own C++ tests:
inputs U(-0.1, 0.1), Linear weights and biases U(-0.02, 0.02), RMSNorm gains
U(0.8, 1.2) (include/tests.h:91-170); N = 37 prefill rows, decode at
position 13 (tests/test_linear.cu:32-78, test_rope.cu:24-59,
test_attn.cu:80-182, test_embedding.cu:26-89).  Widths are reduced where the
full 1536 would make the fixtures large."""
import numpy as np

OP_CASES = {
    "linear_n37": {"kind": "linear", "n": 37, "k": 256, "m": 384},
    "linear_vec": {"kind": "linear_vec", "k": 512, "m": 256},
    "rmsnorm_n37": {"kind": "rmsnorm", "n": 37, "k": 1536},
    "rope_n37": {"kind": "rope", "n": 37, "heads": 24},
    "rope_pos13": {"kind": "rope_vec", "heads": 24, "pos": 13},
    "rope_pos767": {"kind": "rope_vec", "heads": 24, "pos": 767},
    "attn_prefill_n37": {"kind": "attn_prefill", "n": 37, "heads": 4, "max_ctx": 64},
    "attn_decode_n13": {"kind": "attn_decode", "n": 13, "heads": 4, "max_ctx": 64, "pos": 13},
    "embedding": {"kind": "embedding", "vocab": 1000, "k": 256, "n": 37},
    "swiglu_n5": {"kind": "swiglu", "n": 5, "k": 256, "f": 512},
    "swiglu_vec": {"kind": "swiglu", "n": 1, "k": 256, "f": 512},
}


def _u(g, lo, hi, shape):
    return g.uniform(lo, hi, shape).astype(np.float32)


def case_inputs(name: str) -> dict:
    c = OP_CASES[name]
    g = np.random.default_rng(sum(map(ord, name)) * 7919)
    kind = c["kind"]
    if kind in ("linear", "linear_vec"):
        x = _u(g, -0.1, 0.1, (c.get("n", 1), c["k"]) if kind == "linear" else (c["k"],))
        return {"x": x, "w": _u(g, -0.02, 0.02, (c["m"], c["k"])), "b": _u(g, -0.02, 0.02, (c["m"],))}
    if kind == "rmsnorm":
        return {"x": _u(g, -0.1, 0.1, (c["n"], c["k"])), "gamma": _u(g, 0.8, 1.2, (c["k"],))}
    if kind == "rope":
        return {"x": _u(g, -0.1, 0.1, (c["n"], c["heads"], 64))}
    if kind == "rope_vec":
        return {"x": _u(g, -0.1, 0.1, (c["heads"], 64))}
    if kind == "attn_prefill":
        return {k: _u(g, -0.1, 0.1, (c["n"], c["heads"], 64)) for k in ("q", "k", "v")}
    if kind == "attn_decode":
        kc = np.zeros((c["max_ctx"], c["heads"], 64), np.float32)
        vc = np.zeros_like(kc)
        kc[: c["n"]] = _u(g, -0.1, 0.1, (c["n"], c["heads"], 64))
        vc[: c["n"]] = _u(g, -0.1, 0.1, (c["n"], c["heads"], 64))
        d = {k: _u(g, -0.1, 0.1, (c["heads"], 64)) for k in ("q", "k", "v")}
        d.update(kc=kc, vc=vc)
        return d
    if kind == "embedding":
        return {"table": _u(g, -0.02, 0.02, (c["vocab"], c["k"])),
                "ids": g.integers(0, c["vocab"], c["n"]).astype(np.int32), "h": _u(g, -0.1, 0.1, (c["k"],))}
    if kind == "swiglu":
        k, f, n = c["k"], c["f"], c["n"]
        x = _u(g, -0.1, 0.1, (n, k) if n > 1 else (k,))
        return {"x": x, "w1": _u(g, -0.02, 0.02, (f, k)), "b1": _u(g, -0.02, 0.02, (f,)),
                "v": _u(g, -0.02, 0.02, (f, k)), "bv": _u(g, -0.02, 0.02, (f,)),
                "w2": _u(g, -0.02, 0.02, (k, f)), "b2": _u(g, -0.02, 0.02, (k,))}
    raise ValueError(kind)


# sample_cpu cases: logits ~ N(0, 1.2) over the full vocabulary (the probed
# logit range of the random-weight model is about [-3.6, 3.75]).
SAMPLER_CASES = {
    "greedy": {"seed": 1, "T": 0.7, "p": 0.0, "rp": 1.0, "rep": [], "mt_seed": 5},
    "default": {"seed": 2, "T": 0.7, "p": 0.9, "rp": 1.1, "rep": [3, 99, 151000], "mt_seed": 6},
    "hot": {"seed": 3, "T": 1.5, "p": 0.95, "rp": 1.3, "rep": list(range(0, 600, 7)), "mt_seed": 7},
    "cold": {"seed": 4, "T": 0.1, "p": 0.5, "rp": 1.0, "rep": [], "mt_seed": 8},
    "all1024": {"seed": 5, "T": 0.7, "p": 1.0, "rp": 1.1, "rep": [10], "mt_seed": 9},
    "ties": {"seed": 6, "T": 0.7, "p": 0.9, "rp": 1.0, "rep": [], "mt_seed": 10, "ties": True},
}


def sampler_logits(c: dict) -> np.ndarray:
    g = np.random.default_rng(c["seed"])
    lg = (g.standard_normal(151669) * 1.2).astype(np.float32)
    if c.get("ties"):
        lg[[11, 12, 13]] = lg.max() + 0.5  # an exact three-way tie at the top
    return lg
