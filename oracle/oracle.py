"""Test infrastructure only: ctypes access to the two CPU checkers.

* ``Port`` — the plain-C restatement of the reference's fp32 CPU path
  (oracle/xl_oracle.c -> oracle/_build/libxloracle.so).  The parity checker
  used by tests/ and smoke() on the GPU machine.
* ``Ref``  — the reference engine's own CPU path compiled from its sources
  (oracle/ref_harness.cpp + the reference's src/*.cu -> oracle/_ref/libxlref.so).
  Used here to pin the port (tests/test_oracle_pin.py, tests/golden/) and by
  bench.py as the timed reference CPU baseline.  Processes that load it
  should run with CUDA_VISIBLE_DEVICES="" (the reference's Tensor mirrors every
  buffer on GPU 0 when a GPU is visible).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm import this module.  The product (xingling-cpp_b200/) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "_build", "libxloracle.so")
REF_SO = os.path.join(HERE, "_ref", "libxlref.so")
# The reference checkout: XL_REFERENCE_SRC, else the directory `reference`
# beside this repository's root.
REFERENCE_SRC = os.environ.get("XL_REFERENCE_SRC",
                               os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))

_f = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build(ref: bool | None = None) -> None:
    """Build the port (always) and the reference harness when its sources exist."""
    subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
    if ref is None:
        ref = os.path.isdir(os.path.join(REFERENCE_SRC, "src"))
    if ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REFERENCE_SRC}"], check=True)


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def _as_f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _as_i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


# ---------------------------------------------------------------------------
class _PortLib:
    _lib = None

    @classmethod
    def get(cls) -> C.CDLL:
        if cls._lib is None:
            if not os.path.exists(PORT_SO):
                build(ref=False)
            lib = C.CDLL(PORT_SO)
            lib.xlo_linear.argtypes = [_f, _f, _f, _f, C.c_int, C.c_int, C.c_int]
            lib.xlo_rmsnorm.argtypes = [_f, _f, C.c_int, C.c_int]
            lib.xlo_rope.argtypes = [_f, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
            lib.xlo_attn_prefill.argtypes = [_f, _f, _f, _f, _f, _f, C.c_int, C.c_int, C.c_int]
            lib.xlo_attn_decode.argtypes = [_f, _f, _f, _f, _f, _f, C.c_int, C.c_int, C.c_int]
            lib.xlo_silu_mul.argtypes = [_f, _f, C.c_size_t]
            lib.xlo_embedding.argtypes = [_f, C.c_int, _i, C.c_int, _f]
            lib.xlo_lm_head.argtypes = [_f, _f, _f, C.c_int, C.c_int]
            lib.xlo_sample.argtypes = [_f, C.c_int, C.c_float, C.c_float, C.c_float, _i, C.c_int, C.c_float]
            lib.xlo_sample.restype = C.c_int
            lib.xlo_model_create.argtypes = [C.c_int] * 6 + [C.c_float]
            lib.xlo_model_create.restype = C.c_void_p
            lib.xlo_model_free.argtypes = [C.c_void_p]
            lib.xlo_model_load.argtypes = [C.c_void_p, C.c_char_p]
            lib.xlo_model_prefill.argtypes = [C.c_void_p, _i, C.c_int, _f]
            lib.xlo_model_decode.argtypes = [C.c_void_p, C.c_int, _f]
            lib.xlo_model_n.argtypes = [C.c_void_p]
            lib.xlo_model_kv_copy.argtypes = [C.c_void_p, C.c_int, C.c_int, _f, _f]
            cls._lib = lib
        return cls._lib


class Port:
    """The C restatement, model level (Transformer + KVcache semantics)."""

    def __init__(self, shape):
        self.shape = shape
        self.lib = _PortLib.get()
        self.h = self.lib.xlo_model_create(shape.layers, shape.hidden, shape.heads, shape.ffn, shape.vocab,
                                           shape.max_ctx, shape.rope_base)

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.xlo_model_free(self.h)
            self.h = None

    def load(self, path: str) -> None:
        if self.lib.xlo_model_load(self.h, path.encode()) != 0:
            raise IOError(f"oracle: cannot load weight tree {path}")

    def prefill(self, ids) -> np.ndarray:
        out = np.empty(self.shape.vocab, np.float32)
        rc = self.lib.xlo_model_prefill(self.h, _as_i32(ids), len(ids), out)
        if rc:
            raise ValueError(f"oracle prefill rc={rc}")
        return out

    def decode(self, token: int) -> np.ndarray:
        out = np.empty(self.shape.vocab, np.float32)
        rc = self.lib.xlo_model_decode(self.h, int(token), out)
        if rc:
            raise ValueError(f"oracle decode rc={rc}")
        return out

    @property
    def n(self) -> int:
        return self.lib.xlo_model_n(self.h)

    def kv(self, layer: int, npos: int) -> tuple[np.ndarray, np.ndarray]:
        k = np.empty((npos, self.shape.heads, 64), np.float32)
        v = np.empty_like(k)
        self.lib.xlo_model_kv_copy(self.h, layer, npos, k, v)
        return k, v


# op-level port functions -----------------------------------------------------
def linear(x, w, b) -> np.ndarray:
    x, w, b = _as_f32(x), _as_f32(w), _as_f32(b)
    n, k = x.reshape(-1, x.shape[-1]).shape
    m = w.shape[0]
    out = np.empty((n, m), np.float32)
    _PortLib.get().xlo_linear(x, w, b, out, n, k, m)
    return out.reshape(*x.shape[:-1], m)


def rmsnorm(x, gamma) -> np.ndarray:
    y = _as_f32(x).copy()
    k = y.shape[-1]
    _PortLib.get().xlo_rmsnorm(y, _as_f32(gamma), y.size // k, k)
    return y


def rope(x, start_pos: int, base: float = 10000.0) -> np.ndarray:
    """x: [n][heads][64]; row i is rotated at position start_pos + i."""
    y = _as_f32(x).copy()
    n, heads, c = y.shape
    _PortLib.get().xlo_rope(y, n, heads, c, start_pos, base)
    return y


def attn_prefill(q, k, v, max_ctx: int):
    q, k, v = _as_f32(q), _as_f32(k), _as_f32(v)
    n, heads, c = q.shape
    out = np.empty_like(q)
    kc = np.zeros((max_ctx, heads, c), np.float32)
    vc = np.zeros_like(kc)
    _PortLib.get().xlo_attn_prefill(q, k, v, out, kc, vc, n, heads, c)
    return out, kc, vc


def attn_decode(q, k, v, kc, vc, pos: int):
    """q/k/v: [heads][64]; kc/vc: [max_ctx][heads][64] (copied, then appended at pos)."""
    q, k, v = _as_f32(q), _as_f32(k), _as_f32(v)
    kc, vc = _as_f32(kc).copy(), _as_f32(vc).copy()
    heads, c = q.shape
    out = np.empty_like(q)
    _PortLib.get().xlo_attn_decode(q, k, v, out, kc, vc, pos, heads, c)
    return out, kc, vc


def silu_mul(a, b) -> np.ndarray:
    y = _as_f32(a).copy()
    _PortLib.get().xlo_silu_mul(y, _as_f32(b), y.size)
    return y


def lm_head(table, h) -> np.ndarray:
    table = _as_f32(table)
    out = np.empty(table.shape[0], np.float32)
    _PortLib.get().xlo_lm_head(table, _as_f32(h), out, table.shape[0], table.shape[1])
    return out


def sample(logits, temperature: float, top_p: float, rp: float, rep_ids, r: float) -> int:
    """sample_cpu restated with the uniform r supplied (penalty applied to a copy)."""
    lg = _as_f32(logits).copy()
    rep = _as_i32(sorted(set(int(t) for t in rep_ids)) or [0])
    return int(_PortLib.get().xlo_sample(lg, lg.size, temperature, top_p, rp, rep, len(set(rep_ids)), r))


def apply_penalty(logits, rep_ids, rp: float) -> np.ndarray:
    """The in-place penalty step of sample_cpu (src/inference.cu:71-74), on a copy."""
    lg = _as_f32(logits).copy()
    for t in set(int(x) for x in rep_ids):
        lg[t] = lg[t] / np.float32(rp) if lg[t] > 0 else lg[t] * np.float32(rp)
    return lg


# ---------------------------------------------------------------------------
class _RefLib:
    _lib = None

    @classmethod
    def get(cls) -> C.CDLL:
        if cls._lib is None:
            if not os.path.exists(REF_SO):
                raise FileNotFoundError(f"{REF_SO} is not built (needs the reference sources)")
            lib = C.CDLL(REF_SO)
            lib.xlref_model_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int, C.c_int]
            lib.xlref_model_create.restype = C.c_void_p
            lib.xlref_model_load.argtypes = [C.c_void_p, C.c_char_p]
            lib.xlref_model_prefill.argtypes = [C.c_void_p, _i, C.c_int, _f]
            lib.xlref_model_decode.argtypes = [C.c_void_p, C.c_int, _f]
            lib.xlref_model_kv_n.argtypes = [C.c_void_p, C.c_int]
            lib.xlref_model_kv_copy.argtypes = [C.c_void_p, C.c_int, C.c_int, _f, _f]
            lib.xlref_sample.argtypes = [_f, C.c_int, C.c_float, C.c_float, C.c_float, C.c_uint32, _i, C.c_int]
            lib.xlref_mt_uniform.argtypes = [C.c_uint32]
            lib.xlref_mt_uniform.restype = C.c_float
            lib.xlref_linear.argtypes = [_f, _f, _f, _f, C.c_int, C.c_int, C.c_int, C.c_int]
            lib.xlref_rmsnorm.argtypes = [_f, _f, C.c_int, C.c_int]
            lib.xlref_rope.argtypes = [_f, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
            lib.xlref_attn_prefill.argtypes = [_f, _f, _f, _f, _f, _f, C.c_int, C.c_int, C.c_int, C.c_int]
            lib.xlref_attn_decode.argtypes = [_f, _f, _f, _f, _f, _f, C.c_int, C.c_int, C.c_int, C.c_int]
            lib.xlref_embedding.argtypes = [_f, C.c_int, C.c_int, _i, C.c_int, _f, C.c_void_p, C.c_void_p]
            lib.xlref_swiglu.argtypes = [_f, _f, _f, _f, _f, _f, _f, C.c_int, C.c_int, C.c_int]
            cls._lib = lib
        return cls._lib


class Ref:
    """The reference's own Transformer on its CPU path (objects are leaked by design)."""

    def __init__(self, shape):
        self.shape = shape
        self.lib = _RefLib.get()
        self.h = self.lib.xlref_model_create(shape.max_ctx, shape.hidden, shape.heads, shape.rope_base, shape.ffn,
                                             shape.vocab, shape.layers)

    def load(self, path: str) -> None:
        if self.lib.xlref_model_load(self.h, path.encode()) != 0:
            raise IOError(f"reference: cannot load weight tree {path}")

    def prefill(self, ids) -> np.ndarray:
        out = np.empty(self.shape.vocab, np.float32)
        rc = self.lib.xlref_model_prefill(self.h, _as_i32(ids), len(ids), out)
        if rc:
            raise ValueError(f"reference prefill rc={rc}")
        return out

    def decode(self, token: int) -> np.ndarray:
        out = np.empty(self.shape.vocab, np.float32)
        rc = self.lib.xlref_model_decode(self.h, int(token), out)
        if rc:
            raise ValueError(f"reference decode rc={rc}")
        return out

    def kv_n(self, layer: int) -> int:
        return self.lib.xlref_model_kv_n(self.h, layer)

    def kv(self, layer: int, npos: int) -> tuple[np.ndarray, np.ndarray]:
        k = np.empty((npos, self.shape.heads, 64), np.float32)
        v = np.empty_like(k)
        self.lib.xlref_model_kv_copy(self.h, layer, npos, k, v)
        return k, v


def ref_sample(logits, temperature, top_p, rp, rep_ids, mt_seed: int) -> tuple[int, float]:
    """The reference's sample_cpu with std::mt19937(mt_seed); returns (id, the uniform it drew)."""
    lib = _RefLib.get()
    lg = _as_f32(logits).copy()
    rep = _as_i32(sorted(set(int(t) for t in rep_ids)) or [0])
    tok = lib.xlref_sample(lg, lg.size, temperature, top_p, rp, mt_seed, rep, len(set(rep_ids)))
    return int(tok), float(lib.xlref_mt_uniform(mt_seed))


def ref_linear(x, w, b, vec: bool = False) -> np.ndarray:
    x, w, b = _as_f32(x), _as_f32(w), _as_f32(b)
    k = x.shape[-1]
    n = x.size // k
    m = w.shape[0]
    out = np.empty((n, m), np.float32)
    _RefLib.get().xlref_linear(x, w, b, out, n, k, m, 1 if vec else 0)
    return out.reshape(*x.shape[:-1], m)


def ref_rmsnorm(x, gamma) -> np.ndarray:
    y = _as_f32(x).copy()
    k = y.shape[-1]
    _RefLib.get().xlref_rmsnorm(y, _as_f32(gamma), y.size // k, k)
    return y


def ref_rope(x, pos: int | None, base: float = 10000.0) -> np.ndarray:
    """pos None: RoPE::forward on [n][heads][64]; else RoPE::forward_vec on [heads][64]."""
    y = _as_f32(x).copy()
    if pos is None:
        n, heads, c = y.shape
        _RefLib.get().xlref_rope(y, n, heads, c, -1, base)
    else:
        heads, c = y.shape
        _RefLib.get().xlref_rope(y, 1, heads, c, pos, base)
    return y


def ref_attn_prefill(q, k, v, max_ctx: int):
    q, k, v = _as_f32(q), _as_f32(k), _as_f32(v)
    n, heads, c = q.shape
    out = np.empty_like(q)
    kc = np.zeros((max_ctx, heads, c), np.float32)
    vc = np.zeros_like(kc)
    _RefLib.get().xlref_attn_prefill(q, k, v, out, kc, vc, n, heads, c, max_ctx)
    return out, kc, vc


def ref_attn_decode(q, k, v, kc, vc, pos: int):
    q, k, v = _as_f32(q), _as_f32(k), _as_f32(v)
    kc, vc = _as_f32(kc).copy(), _as_f32(vc).copy()
    heads, c = q.shape
    out = np.empty_like(q)
    _RefLib.get().xlref_attn_decode(q, k, v, out, kc, vc, pos, heads, c, kc.shape[0])
    return out, kc, vc


def ref_embedding(table, ids, h=None):
    table = _as_f32(table)
    vocab, k = table.shape
    ids = _as_i32(ids)
    rows = np.empty((len(ids), k), np.float32)
    logits = np.empty(vocab, np.float32)
    hh = _as_f32(h) if h is not None else None
    _RefLib.get().xlref_embedding(table, vocab, k, ids, len(ids), rows,
                                  hh.ctypes.data if hh is not None else None, logits.ctypes.data)
    return rows, (logits if h is not None else None)


def ref_swiglu(x, w1, b1, v, bv, w2, b2) -> np.ndarray:
    y = _as_f32(x).copy()
    n = 1 if y.ndim == 1 else y.shape[0]
    in_dim = y.shape[-1]
    hidden = w1.shape[0]
    _RefLib.get().xlref_swiglu(y, _as_f32(w1), _as_f32(b1), _as_f32(v), _as_f32(bv), _as_f32(w2), _as_f32(b2), n,
                               in_dim, hidden)
    return y
