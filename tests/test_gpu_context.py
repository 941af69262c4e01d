"""Contexts past the reference's 768 positions and prefill continuation
(InferenceEngine.extend / xl_engine_extend), against the oracle port.

* max_ctx 1536 (tiny shape, both decode paths) and 1024 (the full-width
  2-layer shape, where the persistent kernel no longer fits and the per-op path
  runs): prefill past 768, then decode, logits within 1e-3 of the range.
* extend(B) after a prefill of A equals the oracle's prefill of A + B (the
  continuation attends to every cached position), then decode continues alike;
  the repetition set of the earlier ids is kept (the reference clears it only
  on a new prompt, src/inference.cu:116-136).
"""
import numpy as np
import pytest

import oracle as O
import xl_synth as S

pytestmark = pytest.mark.gpu

GREEDY = dict(top_p=0.0, repetition_penalty=1.0)


@pytest.fixture(scope="module")
def eng_mod(built):
    import llm_cpp_engine

    return llm_cpp_engine


def shape_with_ctx(sh, max_ctx):
    return S.ModelShape(layers=sh.layers, hidden=sh.hidden, heads=sh.heads, ffn=sh.ffn, vocab=sh.vocab,
                        max_ctx=max_ctx)


def close(got, ref, what):
    span = float(ref.max() - ref.min())
    err = float(np.abs(got - ref).max())
    assert err <= 1e-3 * span, f"{what}: max |dlogit| {err:.3e} > 1e-3 x {span:.3f}"


def logits(eng):
    return np.frombuffer(eng.last_logits(), np.float32)


def make(eng_mod, sh, wdir, path, prefill_kernels=0):
    eng = eng_mod.InferenceEngine("cuda", **sh.engine_kwargs())
    eng.set_option("decode_path", path)
    eng.set_option("prefill_gemm", prefill_kernels)
    eng.set_option("prefill_attn", prefill_kernels)
    eng.load(wdir)
    return eng


def decode_alike(eng, port, tok_ref, steps, what):
    for step in range(steps):
        eng.next_token(tok_ref, **GREEDY)  # teacher-forced on the oracle's ids
        ref = port.decode(tok_ref)
        close(logits(eng), ref, f"{what} step {step}")
        tok_ref = int(np.argmax(ref))


@pytest.mark.parametrize("base,max_ctx,n,path", [("TINY", 1536, 1100, 0), ("TINY", 1536, 1100, 1),
                                                 ("WIDE2", 1024, 800, 0)],
                         ids=["tiny1536-persistent", "tiny1536-per_op", "wide1024"])
def test_context_past_768(eng_mod, base, max_ctx, n, path):
    sh = shape_with_ctx(getattr(S, base), max_ctx)
    wdir = S.write_weight_tree(f"/tmp/xl_weights/{base.lower()}", getattr(S, base))
    eng = make(eng_mod, sh, wdir, path)
    port = O.Port(sh)
    port.load(wdir)
    ids = S.prompt_ids(8, n, sh.vocab)
    eng.next_token(ids, **GREEDY)
    ref = port.prefill(ids)
    close(logits(eng), ref, "prefill")
    decode_alike(eng, port, int(np.argmax(ref)), 6, "decode")
    assert eng.ctx_len() == n + 6


@pytest.mark.parametrize("path", [0, 1], ids=["persistent", "per_op"])
@pytest.mark.parametrize("prefill_kernels", [0, 1], ids=["tcgen05", "fma"])
def test_extend_equals_prefill_of_the_concatenation(eng_mod, tiny_weights, path, prefill_kernels):
    sh = S.TINY
    eng = make(eng_mod, sh, tiny_weights, path, prefill_kernels)
    port = O.Port(sh)
    port.load(tiny_weights)
    a = S.prompt_ids(11, 70, sh.vocab)
    b = S.prompt_ids(12, 45, sh.vocab)
    eng.next_token(a, **GREEDY)
    for rnd in range(2):  # a second continuation on top of the first
        eng.extend(b, **GREEDY)
        ref = port.prefill(a + b * (rnd + 1))
        close(logits(eng), ref, f"extend {rnd}")
        assert eng.ctx_len() == len(a) + len(b) * (rnd + 1)
    decode_alike(eng, port, int(np.argmax(ref)), 8, "after extend")


def test_extend_keeps_the_repetition_set(eng_mod, tiny_weights):
    sh = S.TINY
    eng = make(eng_mod, sh, tiny_weights, 0)
    port = O.Port(sh)
    port.load(tiny_weights)
    a = S.prompt_ids(13, 40, sh.vocab)
    b = S.prompt_ids(14, 20, sh.vocab)
    rp = 1.3
    t = eng.next_token(a, top_p=0.0, repetition_penalty=rp)  # t enters the set
    eng.extend(b, top_p=0.0, repetition_penalty=rp)
    ref = O.apply_penalty(port.prefill(a + b), [t], rp)
    close(logits(eng), ref, "extend with the earlier id penalised")


def test_extend_errors(eng_mod, tiny_weights):
    sh = S.TINY
    eng = make(eng_mod, sh, tiny_weights, 0)
    with pytest.raises(RuntimeError):
        eng.extend([1, 2, 3])  # nothing cached yet
    eng.next_token(S.prompt_ids(15, sh.max_ctx - 4, sh.vocab), **GREEDY)
    with pytest.raises(RuntimeError):
        eng.extend([1, 2, 3, 4, 5], **GREEDY)  # past the context
    eng.extend([1, 2, 3, 4], **GREEDY)
    assert eng.ctx_len() == sh.max_ctx
