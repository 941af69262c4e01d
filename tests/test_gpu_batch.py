"""Batched decode (llm_cpp_engine.BatchDecoder, xl_batch_* in the C ABI): eight
sequences with different prompts decode together over one engine's weights.
Every sequence is checked against its own oracle port on the same weights:

* greedy, teacher-forced on the oracle's ids: logits within 1e-3 of their
  range every step, ids equal to the oracle's argmax except at near-ties;
* sampled (temperature 0.7, top_p 0.9, repetition penalty 1.1, a Philox stream
  per sequence): each id is exactly sample_cpu's draw on that sequence's
  penalised logits with that sequence's uniform, and the logits match the
  oracle's penalised with the sequence's own history.
"""
import numpy as np
import pytest

import oracle as O
import xl_synth as S

pytestmark = pytest.mark.gpu

B = 8


@pytest.fixture(scope="module")
def eng_mod(built):
    import llm_cpp_engine

    return llm_cpp_engine


def close(got, ref, what):
    span = float(ref.max() - ref.min())
    err = float(np.abs(got - ref).max())
    assert err <= 1e-3 * span, f"{what}: max |dlogit| {err:.3e} > 1e-3 x {span:.3f}"


def token_ok(tok, ref, what):
    want = int(np.argmax(ref))
    if tok != want:
        a = np.partition(ref, -2)[-2:]
        assert a[1] - a[0] < 1e-3 * float(ref.max() - ref.min()), f"{what}: {tok} != oracle {want}"


def logits_of(bd, seq, vocab):
    return np.frombuffer(bd.last_logits(seq, vocab), np.float32)


PATHS = pytest.mark.parametrize("path", [0, 1], ids=["persistent", "per_op"])  # 0: batch_persistent 1


def greedy_launches(path, sh):
    # persistent: the step inputs + one batched persistent kernel (it writes the greedy ids);
    # per-op: inputs, six kernels per layer, the LM head and the greedy finish
    return 2 if path == 0 else 1 + 6 * sh.layers + 2


def sampled_launches(path, sh):
    return (2 if path == 0 else 1 + 6 * sh.layers + 1) + 4  # ... then the sampler chain


@PATHS
@pytest.mark.parametrize("shape_name,steps", [("TINY", 6), ("WIDE2", 3)])
def test_batch_greedy_matches_oracle_per_sequence(eng_mod, shape_name, steps, path):
    sh = getattr(S, shape_name)
    wdir = S.write_weight_tree(f"/tmp/xl_weights/{shape_name.lower()}", sh)
    eng = eng_mod.InferenceEngine("cuda", **sh.engine_kwargs())
    eng.set_option("decode_path", path)  # the batched decoder follows the engine's decode path
    eng.set_option("batch_persistent", 1 if path == 0 else 0)
    eng.load(wdir)
    bd = eng_mod.BatchDecoder(eng)
    assert eng_mod.BatchDecoder.size == B
    ports, teach = [], []
    for b in range(B):
        ids = S.prompt_ids(100 + b, 5 + 9 * b, sh.vocab)
        tok = bd.prefill(b, ids, temperature=0.7, top_p=0.0, repetition_penalty=1.0)
        port = O.Port(sh)
        port.load(wdir)
        ref = port.prefill(ids)
        close(np.frombuffer(eng.last_logits(), np.float32), ref, f"seq {b} prefill")
        token_ok(tok, ref, f"seq {b} prefill")
        ports.append(port)
        teach.append(int(np.argmax(ref)))
        assert bd.ctx_len(b) == len(ids)
    for step in range(steps):
        n0 = eng_mod.kernel_launches()
        out = bd.step(teach, temperature=0.7, top_p=0.0, repetition_penalty=1.0)
        assert eng_mod.kernel_launches() - n0 == greedy_launches(path, sh)
        nxt = []
        for b in range(B):
            ref = ports[b].decode(teach[b])
            close(logits_of(bd, b, sh.vocab), ref, f"seq {b} step {step}")
            token_ok(out[b], ref, f"seq {b} step {step}")
            nxt.append(int(np.argmax(ref)))
        teach = nxt
    for b in range(B):
        assert bd.ctx_len(b) == 5 + 9 * b + steps


@PATHS
def test_batch_sampled_draws_match_sample_cpu(eng_mod, path):
    sh = S.TINY
    wdir = S.write_weight_tree("/tmp/xl_weights/tiny", sh)
    eng = eng_mod.InferenceEngine("cuda", **sh.engine_kwargs())
    eng.set_option("decode_path", path)
    eng.set_option("batch_persistent", 1 if path == 0 else 0)
    eng.load(wdir)
    bd = eng_mod.BatchDecoder(eng)
    T, P, RP = 0.7, 0.9, 1.1
    seeds = [7000 + 13 * b for b in range(B)]
    ports, hist, toks = [], [], []
    for b in range(B):
        bd.seed(b, seeds[b])
        ids = S.prompt_ids(200 + b, 11 + 3 * b, sh.vocab)
        tok = bd.prefill(b, ids, temperature=T, top_p=P, repetition_penalty=RP)
        u0 = float(S.philox_uniforms(seeds[b], 1, 0)[0])
        assert tok == O.sample(np.frombuffer(eng.last_logits(), np.float32), T, P, 1.0, [], u0)
        port = O.Port(sh)
        port.load(wdir)
        port.prefill(ids)
        ports.append(port)
        hist.append([tok])
        toks.append(tok)
    for step in range(5):
        n0 = eng_mod.kernel_launches()
        out = bd.step(toks, temperature=T, top_p=P, repetition_penalty=RP)
        assert eng_mod.kernel_launches() - n0 == sampled_launches(path, sh)
        for b in range(B):
            got = logits_of(bd, b, sh.vocab)
            u = float(S.philox_uniforms(seeds[b], 1, step + 1)[0])
            assert out[b] == O.sample(got, T, P, 1.0, [], u), f"seq {b} step {step}: draw differs from sample_cpu"
            ref = O.apply_penalty(ports[b].decode(toks[b]), hist[b], RP)
            close(got, ref, f"seq {b} step {step}")
            hist[b].append(out[b])
        toks = list(out)


@PATHS
def test_batch_full_model_greedy(eng_mod, full_weights, path):
    """XingLing-0.68B, eight prompts with lengths drawn like the replica workload
    (uniform in [16, 512], seed 5), four greedy batched steps.  Each sequence is
    then replayed on one oracle port: the prefill and every step's logits on the
    same history (the ids the batch fed itself) within 1e-3 of their range, and
    every id the oracle's argmax except at near-ties."""
    sh = S.FULL
    eng = eng_mod.InferenceEngine("cuda")
    eng.set_option("decode_path", path)
    eng.set_option("batch_persistent", 1 if path == 0 else 0)
    eng.load(full_weights)
    bd = eng_mod.BatchDecoder(eng)
    lens = np.random.default_rng(5).integers(16, 513, B)
    prompts = [S.prompt_ids(500 + b, int(lens[b]), sh.vocab) for b in range(B)]
    first, pre_logits = [], []
    for b in range(B):
        first.append(bd.prefill(b, prompts[b], top_p=0.0, repetition_penalty=1.0))
        pre_logits.append(np.frombuffer(eng.last_logits(), np.float32).copy())
    steps, toks, logits = 4, [first], []
    for _ in range(steps):
        out = bd.step(toks[-1], top_p=0.0, repetition_penalty=1.0)
        logits.append([logits_of(bd, b, sh.vocab).copy() for b in range(B)])
        toks.append(list(out))
    port = O.Port(sh)
    port.load(full_weights)
    for b in range(B):
        ref = port.prefill(prompts[b])
        close(pre_logits[b], ref, f"seq {b} prefill")
        token_ok(toks[0][b], ref, f"seq {b} prefill")
        for step in range(steps):
            ref = port.decode(toks[step][b])
            close(logits[step][b], ref, f"seq {b} step {step}")
            token_ok(toks[step + 1][b], ref, f"seq {b} step {step}")
        assert bd.ctx_len(b) == int(lens[b]) + steps


def test_batch_requires_prefill_and_checks_ids(eng_mod):
    sh = S.TINY
    wdir = S.write_weight_tree("/tmp/xl_weights/tiny", sh)
    eng = eng_mod.InferenceEngine("cuda", **sh.engine_kwargs())
    eng.load(wdir)
    bd = eng_mod.BatchDecoder(eng)
    with pytest.raises(RuntimeError):
        bd.step([1] * B)  # no prompts yet
    for b in range(B):
        bd.prefill(b, [1, 2, 3], top_p=0.0)
    with pytest.raises(ValueError):
        bd.step([1] * (B - 1))
    with pytest.raises(ValueError):
        bd.step([sh.vocab] + [1] * (B - 1))
