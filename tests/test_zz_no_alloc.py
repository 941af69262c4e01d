"""The allocation-free decode attention entry point, xl_op_attn_decode_noalloc.

It exists for callers that cannot call cudaMalloc on the decode path (an
embedder whose device memory belongs to a pool it must not bypass, or a
latency-critical caller that cannot afford an allocation that may synchronize
the device): its split-K scratch is a static device array inside the library.
This test calls it through the C ABI twice in a row (the shared scratch keeps
the last call's contents, so the second call checks that the counters are
cleared) and checks both results against the workspace entry point
xl_op_attn_decode on the same inputs, within the attention tolerance of
tests/test_gpu_ops.py.  The file is named to be collected last, so that a run
stopping at the first failure has already run every other test."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import xl_capi as X

pytestmark = pytest.mark.gpu

HEADS, T = 24, 768


def _close(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    err = np.abs(a - b)
    assert np.all(err <= 2e-6 + 1e-4 * np.maximum(np.abs(a), np.abs(b))), f"max abs err {err.max():.3e}"


def test_attn_decode_noalloc_matches_workspace_entry(built):
    import torch

    g = np.random.default_rng(2024)
    tab = np.empty(T * 64, np.float32)
    X.check(X.lib().xl_rope_table(10000.0, T, tab.ctypes.data))
    rope = torch.from_numpy(tab).cuda()
    kc0 = torch.zeros((HEADS, T, 64), device="cuda")
    vc0 = torch.zeros((HEADS, T, 64), device="cuda")
    for pos_v in (200, 437):  # two calls in a row, the second at a longer context
        kc0[:, :pos_v] = torch.from_numpy(g.uniform(-0.5, 0.5, (HEADS, pos_v, 64)).astype(np.float32)).cuda()
        vc0[:, :pos_v] = torch.from_numpy(g.uniform(-0.5, 0.5, (HEADS, pos_v, 64)).astype(np.float32)).cuda()
        qkv = torch.from_numpy(g.uniform(-0.5, 0.5, 3 * HEADS * 64).astype(np.float32)).cuda()
        pos = torch.tensor([pos_v], dtype=torch.int32, device="cuda")
        ws = torch.zeros(X.lib().xl_op_attn_decode_workspace_bytes(HEADS, T), dtype=torch.uint8, device="cuda")
        kc_a, vc_a, out_a = kc0.clone(), vc0.clone(), torch.empty(HEADS * 64, device="cuda")
        kc_b, vc_b, out_b = kc0.clone(), vc0.clone(), torch.empty(HEADS * 64, device="cuda")
        X.check(X.lib().xl_op_attn_decode(X.ptr(qkv), X.ptr(rope), X.ptr(kc_a), X.ptr(vc_a), X.ptr(out_a),
                                          X.ptr(pos), HEADS, T, X.ptr(ws), X.stream()))
        X.check(X.lib().xl_op_attn_decode_noalloc(X.ptr(qkv), X.ptr(rope), X.ptr(kc_b), X.ptr(vc_b), X.ptr(out_b),
                                                  X.ptr(pos), HEADS, T, X.stream()))
        torch.cuda.synchronize()
        _close(out_b.cpu().numpy(), out_a.cpu().numpy())
        assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)


def test_attn_decode_noalloc_at_the_static_limits_matches_oracle(built):
    """heads 32 and max_ctx 1024 fill the static array exactly (16 splits of
    66 floats per head, then the counters); the last position, 1023, uses every
    split.  Two calls in a row against the oracle's RoPE + KV append + attention
    (src/rope.cu:130-165, src/attn.cu:490-547)."""
    import torch

    heads, t = 32, 1024
    g = np.random.default_rng(77)
    tab = np.empty(t * 64, np.float32)
    X.check(X.lib().xl_rope_table(10000.0, t, tab.ctypes.data))
    rope = torch.from_numpy(tab).cuda()
    for n_prev in (1023, 1000):
        kc_pm = np.zeros((t, heads, 64), np.float32)
        vc_pm = np.zeros((t, heads, 64), np.float32)
        kc_pm[:n_prev] = g.uniform(-0.5, 0.5, (n_prev, heads, 64))
        vc_pm[:n_prev] = g.uniform(-0.5, 0.5, (n_prev, heads, 64))
        q, k, v = (g.uniform(-0.5, 0.5, (heads, 64)).astype(np.float32) for _ in range(3))
        out_ref, kc_ref, vc_ref = O.attn_decode(O.rope(q[None], n_prev)[0], O.rope(k[None], n_prev)[0], v, kc_pm,
                                                vc_pm, n_prev)
        kc = torch.from_numpy(kc_pm.transpose(1, 0, 2).copy()).cuda()
        vc = torch.from_numpy(vc_pm.transpose(1, 0, 2).copy()).cuda()
        qkv = torch.from_numpy(np.concatenate([q.ravel(), k.ravel(), v.ravel()])).cuda()
        out = torch.empty(heads * 64, device="cuda")
        pos = torch.tensor([n_prev], dtype=torch.int32, device="cuda")
        X.check(X.lib().xl_op_attn_decode_noalloc(X.ptr(qkv), X.ptr(rope), X.ptr(kc), X.ptr(vc), X.ptr(out),
                                                  X.ptr(pos), heads, t, X.stream()))
        torch.cuda.synchronize()
        _close(out.cpu().numpy().reshape(heads, 64), out_ref)
        kc_h = kc.cpu().numpy().transpose(1, 0, 2)
        vc_h = vc.cpu().numpy().transpose(1, 0, 2)
        assert np.abs(kc_h[: n_prev + 1] - kc_ref[: n_prev + 1]).max() <= 1e-5
        assert np.array_equal(vc_h[: n_prev + 1], vc_ref[: n_prev + 1])


def test_attn_decode_noalloc_position_past_the_cache_writes_nan(built):
    """A device position at or past max_ctx is refused by the kernel itself:
    the caches stay untouched and every output is NaN (no synchronizing check
    on the host).  A valid call afterwards still matches the workspace entry."""
    import torch

    g = np.random.default_rng(5)
    tab = np.empty(T * 64, np.float32)
    X.check(X.lib().xl_rope_table(10000.0, T, tab.ctypes.data))
    rope = torch.from_numpy(tab).cuda()
    kc = torch.from_numpy(g.uniform(-0.5, 0.5, (HEADS, T, 64)).astype(np.float32)).cuda()
    vc = torch.from_numpy(g.uniform(-0.5, 0.5, (HEADS, T, 64)).astype(np.float32)).cuda()
    kc0, vc0 = kc.clone(), vc.clone()
    qkv = torch.from_numpy(g.uniform(-0.5, 0.5, 3 * HEADS * 64).astype(np.float32)).cuda()
    out = torch.zeros(HEADS * 64, device="cuda")
    for bad in (T, T + 5):
        pos = torch.tensor([bad], dtype=torch.int32, device="cuda")
        X.check(X.lib().xl_op_attn_decode_noalloc(X.ptr(qkv), X.ptr(rope), X.ptr(kc), X.ptr(vc), X.ptr(out),
                                                  X.ptr(pos), HEADS, T, X.stream()))
        torch.cuda.synchronize()
        assert torch.isnan(out).all()
        assert torch.equal(kc, kc0) and torch.equal(vc, vc0)
    pos = torch.tensor([T - 1], dtype=torch.int32, device="cuda")
    ws = torch.zeros(X.lib().xl_op_attn_decode_workspace_bytes(HEADS, T), dtype=torch.uint8, device="cuda")
    kc_a, vc_a, out_a = kc0.clone(), vc0.clone(), torch.empty(HEADS * 64, device="cuda")
    X.check(X.lib().xl_op_attn_decode(X.ptr(qkv), X.ptr(rope), X.ptr(kc_a), X.ptr(vc_a), X.ptr(out_a), X.ptr(pos),
                                      HEADS, T, X.ptr(ws), X.stream()))
    X.check(X.lib().xl_op_attn_decode_noalloc(X.ptr(qkv), X.ptr(rope), X.ptr(kc), X.ptr(vc), X.ptr(out), X.ptr(pos),
                                              HEADS, T, X.stream()))
    torch.cuda.synchronize()
    _close(out.cpu().numpy(), out_a.cpu().numpy())
    assert torch.equal(kc, kc_a) and torch.equal(vc, vc_a)


def test_attn_decode_noalloc_rejects_sizes_beyond_the_static_scratch(built):
    lib = X.lib()
    dummy = C.c_void_p(16)
    rc = lib.xl_op_attn_decode_noalloc(dummy, dummy, dummy, dummy, dummy, dummy, 33, T, None)
    assert rc == 1 and b"heads must be <= 32" in lib.xl_last_error()
    rc = lib.xl_op_attn_decode_noalloc(dummy, dummy, dummy, dummy, dummy, dummy, HEADS, 1025, None)
    assert rc == 1
