"""Kernel-level parity through the C ABI: each xl_op_* against the oracle port
(oracle/xl_oracle.c) on seeded inputs, mirroring the reference's per-op tests
(tests/test_linear.cu, test_rmsnorm.cu, test_rope.cu, test_attn.cu,
test_embedding.cu, test_swishglu.cu).  Tolerances are written per test; the
reference's own tests allow 1e-3 (linear, norm, rope, KV), 2e-2 (attention)
and 1e-2 (LM head); the bounds here are tighter."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import xl_capi as X

pytestmark = pytest.mark.gpu

H, HEADS, F, T = 1536, 24, 4096, 768


@pytest.fixture(scope="module")
def torch_cuda(built):
    import torch

    torch.cuda.init()
    return torch


def dev(torch, a):
    """A device copy; callers keep the returned tensor referenced until the
    kernel that reads it has finished (the caching allocator reuses freed blocks)."""
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def close(a, b, atol, rtol):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    err = np.abs(a - b)
    tol = atol + rtol * np.maximum(np.abs(a), np.abs(b))
    assert np.all(err <= tol), f"max abs err {err.max():.3e} at {np.unravel_index(err.argmax(), err.shape)}"


def rng(seed):
    return np.random.default_rng(seed)


@pytest.mark.parametrize("m,k", [(3 * H, H), (H, H), (H, F), (4097, H), (576, 192)])
def test_norm_gemv_plain(torch_cuda, m, k):
    torch = torch_cuda
    g = rng(123)
    x = g.uniform(-0.1, 0.1, k).astype(np.float32)
    w = g.uniform(-0.02, 0.02, (m, k)).astype(np.float32)
    b = g.uniform(-0.02, 0.02, m).astype(np.float32)
    gamma = g.uniform(0.8, 1.2, k).astype(np.float32)
    for use_norm in (False, True):
        y = torch.empty(m, device="cuda")
        dx, dw, db, dg = dev(torch, x), dev(torch, w), dev(torch, b), dev(torch, gamma)
        X.check(X.lib().xl_op_norm_gemv(0, X.ptr(dx), X.ptr(dg) if use_norm else None, X.ptr(dw), X.ptr(db),
                                        X.ptr(y), m, k, X.stream()))
        torch.cuda.synchronize()
        xin = O.rmsnorm(x[None], gamma)[0] if use_norm else x
        close(host(y), O.linear(xin[None], w, b)[0], 1e-5, 1e-4)


def test_norm_gemv_swiglu_and_residual(torch_cuda):
    torch = torch_cuda
    g = rng(456)
    x = g.uniform(-0.1, 0.1, H).astype(np.float32)
    gamma = g.uniform(0.8, 1.2, H).astype(np.float32)
    w1 = g.uniform(-0.02, 0.02, (F, H)).astype(np.float32)
    v = g.uniform(-0.02, 0.02, (F, H)).astype(np.float32)
    b1 = g.uniform(-0.02, 0.02, F).astype(np.float32)
    bv = g.uniform(-0.02, 0.02, F).astype(np.float32)
    w13 = np.empty((2 * F, H), np.float32)
    w13[0::2], w13[1::2] = w1, v
    b13 = np.empty(2 * F, np.float32)
    b13[0::2], b13[1::2] = b1, bv
    y = torch.empty(F, device="cuda")
    dx, dg, dw13, db13 = dev(torch, x), dev(torch, gamma), dev(torch, w13), dev(torch, b13)
    X.check(X.lib().xl_op_norm_gemv(1, X.ptr(dx), X.ptr(dg), X.ptr(dw13), X.ptr(db13), X.ptr(y), 2 * F, H,
                                    X.stream()))
    torch.cuda.synchronize()
    xn = O.rmsnorm(x[None], gamma)
    ref = O.silu_mul(O.linear(xn, w1, b1), O.linear(xn, v, bv))[0]
    close(host(y), ref, 1e-5, 1e-4)
    # residual: y += W2 . h + b2
    w2 = g.uniform(-0.02, 0.02, (H, F)).astype(np.float32)
    b2 = g.uniform(-0.02, 0.02, H).astype(np.float32)
    resid = g.uniform(-1, 1, H).astype(np.float32)
    yr, dw2, db2 = dev(torch, resid), dev(torch, w2), dev(torch, b2)
    X.check(X.lib().xl_op_norm_gemv(2, X.ptr(y), None, X.ptr(dw2), X.ptr(db2), X.ptr(yr), H, F, X.stream()))
    torch.cuda.synchronize()
    close(host(yr), resid + O.linear(ref[None], w2, b2)[0], 1e-5, 1e-4)


def _rope_dev(torch, max_ctx=T):
    tab = np.empty(max_ctx * 64, np.float32)
    X.check(X.lib().xl_rope_table(10000.0, max_ctx, tab.ctypes.data))
    return dev(torch, tab)


@pytest.mark.parametrize("n_prev", [0, 13, 63, 64, 200, 767])
def test_attn_decode(torch_cuda, n_prev):
    """RoPE at position n + KV append + attention over 0..n (test_attn.cu:125-182 uses n = 13)."""
    torch = torch_cuda
    g = rng(1000 + n_prev)
    kc_pm = np.zeros((T, HEADS, 64), np.float32)
    vc_pm = np.zeros((T, HEADS, 64), np.float32)
    kc_pm[:n_prev] = g.uniform(-0.5, 0.5, (n_prev, HEADS, 64))
    vc_pm[:n_prev] = g.uniform(-0.5, 0.5, (n_prev, HEADS, 64))
    q, k, v = (g.uniform(-0.5, 0.5, (HEADS, 64)).astype(np.float32) for _ in range(3))
    # oracle: RoPE::forward_vec on q and k at pos n, then MultiHeadAttention::forward
    qr = O.rope(q[None], n_prev)[0]
    kr = O.rope(k[None], n_prev)[0]
    out_ref, kc_ref, vc_ref = O.attn_decode(qr, kr, v, kc_pm, vc_pm, n_prev)
    # device: head-major cache
    kc = dev(torch, kc_pm.transpose(1, 0, 2).copy())
    vc = dev(torch, vc_pm.transpose(1, 0, 2).copy())
    qkv = dev(torch, np.concatenate([q.ravel(), k.ravel(), v.ravel()]))
    out = torch.empty(HEADS * 64, device="cuda")
    pos = torch.tensor([n_prev], dtype=torch.int32, device="cuda")
    ws = torch.zeros(X.lib().xl_op_attn_decode_workspace_bytes(HEADS, T), dtype=torch.uint8, device="cuda")
    rope = _rope_dev(torch)
    for _ in range(2):  # the workspace must come back zeroed and reusable
        kc_run, vc_run = kc.clone(), vc.clone()
        X.check(X.lib().xl_op_attn_decode(X.ptr(qkv), X.ptr(rope), X.ptr(kc_run), X.ptr(vc_run), X.ptr(out),
                                          X.ptr(pos), HEADS, T, X.ptr(ws), X.stream()))
        torch.cuda.synchronize()
        close(host(out).reshape(HEADS, 64), out_ref, 2e-6, 1e-4)
        kc_h = host(kc_run).transpose(1, 0, 2)
        vc_h = host(vc_run).transpose(1, 0, 2)
        close(kc_h[: n_prev + 1], kc_ref[: n_prev + 1], 1e-6, 1e-5)
        assert np.array_equal(vc_h[: n_prev + 1], vc_ref[: n_prev + 1])  # V append is a copy
        assert not np.any(kc_h[n_prev + 1:]) and not np.any(vc_h[n_prev + 1:])
    assert int(host(ws).astype(np.int64)[-HEADS * 4:].sum()) == 0


@pytest.mark.parametrize("vocab,rp", [(151669, 1.0), (151669, 1.1), (4099, 1.3)])
def test_lm_head(torch_cuda, vocab, rp):
    torch = torch_cuda
    g = rng(789)
    table = (g.standard_normal((vocab, H), dtype=np.float32) * np.float32(0.02))
    x = g.uniform(-1, 1, H).astype(np.float32)
    gamma = np.ones(H, np.float32)
    rep = g.choice(vocab, 40, replace=False)
    flags = np.zeros(vocab, np.uint8)
    flags[rep] = 1
    dt, dx, dgm = dev(torch, table), dev(torch, x), dev(torch, gamma)
    logits = torch.empty(vocab, device="cuda")
    ws = torch.zeros(X.lib().xl_op_lm_head_workspace_bytes(), dtype=torch.uint8, device="cuda")
    arg = C.c_int(-1)
    dflags = dev(torch, flags)
    X.check(X.lib().xl_op_lm_head(X.ptr(dx), X.ptr(dgm), X.ptr(dt), X.ptr(logits), X.ptr(dflags), rp, vocab, H,
                                  C.byref(arg), X.ptr(ws), X.stream()))
    torch.cuda.synchronize()
    ref = O.apply_penalty(O.lm_head(table, O.rmsnorm(x[None], gamma)[0]), rep, rp)
    got = host(logits)
    close(got, ref, 1e-5, 1e-4)
    assert arg.value == int(np.argmax(got))


@pytest.mark.parametrize("temperature,top_p,r", [(0.7, 0.9, 0.3), (0.7, 0.9, 0.999), (1.0, 0.5, 0.01),
                                                 (0.7, 0.0, 0.5), (0.2, 1.0, 0.77)])
def test_sample(torch_cuda, temperature, top_p, r):
    torch = torch_cuda
    g = rng(31)
    logits = (g.standard_normal(151669) * 1.2).astype(np.float32)
    logits[5] = logits[7] = logits.max()  # a tie at the top: lower id first
    dl = dev(torch, logits)
    ws = torch.zeros(X.lib().xl_op_sample_workspace_bytes(151669), dtype=torch.uint8, device="cuda")
    tok = C.c_int(-1)
    X.check(X.lib().xl_op_sample(X.ptr(dl), 151669, temperature, top_p, r, C.byref(tok), X.ptr(ws), X.stream()))
    assert tok.value == O.sample(logits, temperature, top_p, 1.0, [], r)


def sample_logits(dist, g):
    """Logit vectors that drive each branch of the sampler's candidate select."""
    n = 151669
    if dist == "ties_in_window":  # 0.1 steps: a few hundred ids tie at the 1024th value
        return (np.round(g.standard_normal(n) * 1.2, 1)).astype(np.float32)
    if dist == "wide_tie":  # integers: ~9000 ids tie at the threshold (ordered collection)
        return np.round(g.standard_normal(n)).astype(np.float32)
    if dist == "constant":  # every id ties: the 1024 lowest ids are the candidates
        return np.full(n, 0.5, np.float32)
    if dist in ("signed_zeros", "signed_zeros_wide"):  # +0.0 and -0.0 compare equal, lower id first
        x = (np.float32(-1.0) - g.random(n).astype(np.float32)).astype(np.float32)
        ids = g.permutation(n)
        nz = 2000 if dist == "signed_zeros" else 20000
        x[ids[:nz]] = np.where(g.random(nz) < 0.5, np.float32(0.0), np.float32(-0.0))
        x[ids[nz:nz + 900]] = 5.0
        return x
    if dist == "narrow":  # one exponent bin: the first radix pass cannot narrow
        return (np.float32(10.0) + g.standard_normal(n).astype(np.float32) * np.float32(1e-3)).astype(np.float32)
    if dist == "small_vocab":  # fewer ids than candidates
        return (g.standard_normal(700) * 2).astype(np.float32)
    if dist == "mid_vocab":  # all ids gathered without a radix pass
        return (g.standard_normal(3000) * 2).astype(np.float32)
    raise ValueError(dist)


@pytest.mark.parametrize("dist", ["ties_in_window", "wide_tie", "constant", "signed_zeros", "signed_zeros_wide",
                                  "narrow", "small_vocab", "mid_vocab"])
def test_sample_select_branches(torch_cuda, dist):
    """The candidate select gathers ids at or above a radix prefix unordered and sorts
    them, or (a tie wider than its buffer) collects them in id order; every branch must
    give sample_cpu's candidate list, ties to the lower id."""
    torch = torch_cuda
    g = rng(41)
    logits = sample_logits(dist, g)
    n = logits.size
    dl = dev(torch, logits)
    ws = torch.zeros(X.lib().xl_op_sample_workspace_bytes(n), dtype=torch.uint8, device="cuda")
    for temperature, top_p, r in [(0.7, 0.9, 0.3), (1.0, 1.0, 0.999), (0.5, 0.95, 0.61), (1.0, 1.0, 0.0)]:
        tok = C.c_int(-1)
        X.check(X.lib().xl_op_sample(X.ptr(dl), n, temperature, top_p, r, C.byref(tok), X.ptr(ws), X.stream()))
        assert tok.value == O.sample(logits, temperature, top_p, 1.0, [], r), (dist, temperature, top_p, r)


@pytest.mark.parametrize("tensor_cores", [True, False], ids=["tcgen05_3xtf32", "fp32_fma"])
@pytest.mark.parametrize("mode,n,m,k", [(0, 37, H, H), (0, 512, 3 * H, H), (2, 37, H, F), (1, 77, 2 * F, H),
                                        (0, 5, 576, 192), (2, 130, 200, 64)])
def test_linear_prefill(torch_cuda, mode, n, m, k, tensor_cores):
    """Linear::forward at N=37 as tests/test_linear.cu:32-54, plus the fused epilogues; the
    tensor-core path (3xTF32) must keep fp32-level accuracy."""
    torch = torch_cuda
    g = rng(123 + n)
    x = g.uniform(-0.1, 0.1, (n, k)).astype(np.float32)
    w = g.uniform(-0.02, 0.02, (m, k)).astype(np.float32)
    b = g.uniform(-0.02, 0.02, m).astype(np.float32)
    width = m // 2 if mode == 1 else m
    init = g.uniform(-1, 1, (n, width)).astype(np.float32)
    y, dx, dw, db = dev(torch, init), dev(torch, x), dev(torch, w), dev(torch, b)
    x_lo = w_lo = y_lo = None
    if tensor_cores:
        x_lo, w_lo = torch.empty_like(dx), torch.empty_like(dw)
        y_lo = torch.full_like(y, np.nan)
        X.check(X.lib().xl_op_split_lo(X.ptr(dx), X.ptr(x_lo), dx.numel(), X.stream()))
        X.check(X.lib().xl_op_split_lo(X.ptr(dw), X.ptr(w_lo), dw.numel(), X.stream()))
    X.check(X.lib().xl_op_linear(mode, X.ptr(dx), X.ptr(x_lo), X.ptr(dw), X.ptr(w_lo), X.ptr(db), X.ptr(y),
                                 X.ptr(y_lo), n, m, k, X.stream()))
    torch.cuda.synchronize()
    full = O.linear(x, w, b)
    if mode == 0:
        ref = full
    elif mode == 2:
        ref = init + full
    else:
        ref = O.silu_mul(full[:, 0::2], full[:, 1::2])
    # 3xTF32 keeps the products to ~2^-21 relative; the tensor core's fp32
    # accumulation over K terms adds ~1e-6 x sqrt(K / 1536) absolute here.
    close(host(y), ref, 2e-5 if tensor_cores else 2e-6, 1e-4)
    if tensor_cores and mode == 1:
        hy = host(y)
        trunc = (hy.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
        assert np.array_equal(host(y_lo), hy - trunc)


def test_rmsnorm_rows_and_embedding(torch_cuda):
    torch = torch_cuda
    g = rng(123)
    x = g.uniform(-0.1, 0.1, (37, H)).astype(np.float32)
    gamma = g.uniform(0.8, 1.2, H).astype(np.float32)
    dx, dg = dev(torch, x), dev(torch, gamma)
    out = torch.empty_like(dx)
    X.check(X.lib().xl_op_rmsnorm(X.ptr(dx), X.ptr(dg), X.ptr(out), 37, H, X.stream()))
    torch.cuda.synchronize()
    close(host(out), O.rmsnorm(x, gamma), 1e-6, 1e-5)
    table = g.uniform(-0.02, 0.02, (5000, H)).astype(np.float32)
    ids = g.integers(0, 5000, 37).astype(np.int32)
    rows = torch.empty((37, H), device="cuda")
    dtab, dids = dev(torch, table), dev(torch, ids)
    X.check(X.lib().xl_op_embedding(X.ptr(dtab), X.ptr(dids), X.ptr(rows), 37, H, X.stream()))
    torch.cuda.synchronize()
    assert np.array_equal(host(rows), table[ids])  # gather is bit-exact


@pytest.mark.parametrize("n", [1, 37, 64, 130, 512])
def test_attn_prefill(torch_cuda, n):
    """RoPE + KV fill + causal attention (tests/test_attn.cu:80-123 uses N = 37)."""
    torch = torch_cuda
    g = rng(2000 + n)
    q, k, v = (g.uniform(-0.5, 0.5, (n, HEADS, 64)).astype(np.float32) for _ in range(3))
    out_ref, kc_ref, vc_ref = O.attn_prefill(O.rope(q, 0), O.rope(k, 0), v, T)
    qkv = dev(torch, np.concatenate([q.reshape(n, -1), k.reshape(n, -1), v.reshape(n, -1)], axis=1))
    kc = torch.zeros((HEADS, T, 64), device="cuda")
    vc = torch.zeros((HEADS, T, 64), device="cuda")
    out = torch.empty((n, H), device="cuda")
    rope = _rope_dev(torch)
    X.check(X.lib().xl_op_attn_prefill(X.ptr(qkv), X.ptr(rope), X.ptr(kc), X.ptr(vc), X.ptr(out), n, HEADS, T,
                                       X.stream()))
    torch.cuda.synchronize()
    close(host(out).reshape(n, HEADS, 64), out_ref, 2e-6, 1e-4)
    close(host(kc).transpose(1, 0, 2)[:n], kc_ref[:n], 1e-6, 1e-5)
    assert np.array_equal(host(vc).transpose(1, 0, 2)[:n], vc_ref[:n])
