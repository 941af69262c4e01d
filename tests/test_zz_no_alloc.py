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


def test_attn_decode_noalloc_rejects_sizes_beyond_the_static_scratch(built):
    lib = X.lib()
    dummy = C.c_void_p(16)
    rc = lib.xl_op_attn_decode_noalloc(dummy, dummy, dummy, dummy, dummy, dummy, 33, T, None)
    assert rc == 1 and b"heads must be <= 32" in lib.xl_last_error()
    rc = lib.xl_op_attn_decode_noalloc(dummy, dummy, dummy, dummy, dummy, dummy, HEADS, 1025, None)
    assert rc == 1
