"""Device-side multi-token loop (InferenceEngine.generate, xl_engine_generate).

generate(token, n) must give the ids, the draws and the engine state that n
successive next_token calls give: the same ids (the decode kernels are
deterministic, so the logits are bit-identical too), the same context length,
one uniform per step taken (unused draws go back to the queue / the Philox
counter), a stop id that ends the run and is returned, and a stop at the full
cache.  The persistent decode path runs the loop on the device (one graph
launch per step: feed, decode step, collect); the per-op path runs it on the
host.
"""
import numpy as np
import pytest

import xl_synth as S

pytestmark = pytest.mark.gpu

PATHS = pytest.mark.parametrize("path", [0, 1], ids=["persistent", "per_op"])
GREEDY = dict(top_p=0.0, repetition_penalty=1.0)
SAMPLED = dict(temperature=0.7, top_p=0.9, repetition_penalty=1.1)


@pytest.fixture(scope="module")
def eng_mod(built):
    import llm_cpp_engine

    return llm_cpp_engine


def engine(mod, weights, path, sh=S.TINY):
    eng = mod.InferenceEngine("cuda", **sh.engine_kwargs())
    eng.set_option("decode_path", path)
    eng.load(weights)
    return eng


def logits(eng):
    return np.frombuffer(eng.last_logits(), np.float32)


@PATHS
@pytest.mark.parametrize("sampled", [False, True], ids=["greedy", "sampled"])
def test_generate_equals_next_token_loop(eng_mod, tiny_weights, path, sampled):
    kw = SAMPLED if sampled else GREEDY
    ids = S.prompt_ids(4, 23, S.TINY.vocab)
    a, b = engine(eng_mod, tiny_weights, path), engine(eng_mod, tiny_weights, path)
    a.seed(11)
    b.seed(11)
    ta, tb = a.next_token(ids, **kw), b.next_token(ids, **kw)
    assert ta == tb
    loop, t = [], ta
    for _ in range(25):
        t = a.next_token(t, **kw)
        loop.append(t)
    gen = b.generate(tb, 25, **kw)
    assert gen == loop
    assert a.ctx_len() == b.ctx_len() == 23 + 25
    assert np.array_equal(logits(a), logits(b))
    assert a.next_token(loop[-1], **kw) == b.next_token(gen[-1], **kw)  # the draws continue alike


def first_new(seq, start):
    """The first index k >= start whose id has not appeared before it."""
    for k in range(start, len(seq)):
        if seq[k] not in seq[:k]:
            return k
    pytest.skip("no fresh id in the sequence")


def test_generate_stop_id_returns_unused_draws(eng_mod, tiny_weights):
    """A stop id ends the run after it; the draws of the steps never taken go
    back (first to the explicit queue, then to the Philox counter), so later
    calls continue exactly as the next_token loop does."""
    ids = S.prompt_ids(5, 17, S.TINY.vocab)
    queued = [float(x) for x in S.philox_uniforms(9, 4)]  # 4 explicit draws, then the Philox stream
    a, b = engine(eng_mod, tiny_weights, 0), engine(eng_mod, tiny_weights, 0)
    for e in (a, b):
        e.seed(21)
        e.set_uniforms(queued)
    ta, tb = a.next_token(ids, **SAMPLED), b.next_token(ids, **SAMPLED)
    assert ta == tb
    seq, t = [], ta
    for _ in range(30):
        t = a.next_token(t, **SAMPLED)
        seq.append(t)
    k = first_new(seq, 1)  # stops after step k (a draw from the queue is left over when k < 2)
    gen = b.generate(tb, 30, stop_id=seq[k], **SAMPLED)
    assert gen == seq[: k + 1]
    assert b.ctx_len() == 17 + k + 1
    rest = b.generate(gen[-1], 30 - k - 1, **SAMPLED)
    assert rest == seq[k + 1:]
    assert b.ctx_len() == a.ctx_len()
    assert np.array_equal(logits(a), logits(b))


@PATHS
def test_generate_stops_at_full_cache(eng_mod, tiny_weights, path):
    sh = S.TINY
    eng = engine(eng_mod, tiny_weights, path)
    t = eng.next_token(S.prompt_ids(6, sh.max_ctx - 8, sh.vocab), **GREEDY)
    out = eng.generate(t, 20, **GREEDY)
    assert len(out) == 8 and eng.ctx_len() == sh.max_ctx
    with pytest.raises(RuntimeError):
        eng.generate(out[-1], 3, **GREEDY)
    assert eng.generate(out[-1], 0, **GREEDY) == []


def test_generate_launches_per_step(eng_mod, tiny_weights):
    """One graph per step: gen_feed, the persistent kernel, gen_collect (greedy);
    the sampled graph adds the sampler chain (3 histogram passes + gather)."""
    eng = engine(eng_mod, tiny_weights, 0)
    t = eng.next_token(S.prompt_ids(7, 9, S.TINY.vocab), **GREEDY)
    n0 = eng_mod.kernel_launches()
    out = eng.generate(t, 10, **GREEDY)
    assert len(out) == 10 and eng_mod.kernel_launches() - n0 == 10 * 3
    n0 = eng_mod.kernel_launches()
    eng.generate(out[-1], 6, **SAMPLED)
    assert eng_mod.kernel_launches() - n0 == 6 * 7


def test_generate_full_model_greedy(eng_mod, full_weights):
    """XingLing-0.68B: 40 ids from one device-side loop equal 40 next_token calls."""
    ids = S.prompt_ids(0, 32, S.FULL.vocab)
    a, b = engine(eng_mod, full_weights, 0, S.FULL), engine(eng_mod, full_weights, 0, S.FULL)
    ta, tb = a.next_token(ids, **GREEDY), b.next_token(ids, **GREEDY)
    loop, t = [], ta
    for _ in range(40):
        t = a.next_token(t, **GREEDY)
        loop.append(t)
    assert b.generate(tb, 40, **GREEDY) == loop
    assert np.array_equal(logits(a), logits(b))
