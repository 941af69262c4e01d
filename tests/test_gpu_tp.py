"""Tensor-parallel decode on two GPUs (skipped with fewer): two spawned ranks,
each one shard of the engine on its own GPU with the engine's own NCCL
communicator (rank 0's id handed over through a queue), against the oracle
port on the same weight tree.

Both decode paths: the persistent kernel (the out-projection and W2 partial
sums of every CTA go to every rank's exchange buffer over NVLink and each
rank sums them in the same order; one kernel + the greedy finish per step;
TINY's shards stream as k-tiles of 128 floats) and the per-op path (NCCL
all-reduces).

* Greedy, teacher-forced on the oracle's ids: the ranks' vocab shards,
  concatenated, match the oracle's logits within 1e-3 of their range, and
  every rank returns the same id (the greedy merge of per-shard maxima).
* Sampled (temperature 0.7, top_p 0.9, repetition penalty 1.1, the same
  Philox uniforms queued on both ranks), free-running: every rank returns the
  same id, which is exactly sample_cpu's draw on the concatenated penalised
  logits (the all-gather merge of per-shard top-1024 lists), and those logits
  match the oracle's, penalised with the engine's own history, within 1e-3 of
  their range.

NVLS stays off: a rank that fails must not leave memory bound to an NVLink
multicast object."""
import os
import queue
import sys

import numpy as np
import pytest

import oracle as O
import xl_synth as S

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORLD = 2


def _gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _rank(rank, world, wdir, shape_kw, ids, teach, q_id, q_out, sampled=None, path=0):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path[:0] = [os.path.join(ROOT, "xingling-cpp_b200")]
    try:
        import llm_cpp_engine as m

        if rank == 0:
            ident = m.nccl_unique_id()
            for _ in range(world - 1):
                q_id.put(ident)
        else:
            ident = q_id.get(timeout=120)
        eng = m.InferenceEngine(f"cuda:{rank}", tp=world, rank=rank, nccl_id=ident, **shape_kw)
        eng.set_option("decode_path", path)
        eng.load(wdir)
        toks, logits = [], []
        step_launches = 0
        if sampled is None:
            tok = eng.next_token(ids, top_p=0.0, repetition_penalty=1.0)
            toks.append(tok)
            logits.append(np.frombuffer(eng.last_logits(), np.float32).copy())
            for t in teach:
                n0 = m.kernel_launches()
                tok = eng.next_token(int(t), top_p=0.0, repetition_penalty=1.0)
                step_launches = m.kernel_launches() - n0
                toks.append(tok)
                logits.append(np.frombuffer(eng.last_logits(), np.float32).copy())
        else:
            T, P, RP, uniforms = sampled
            eng.set_uniforms([float(u) for u in uniforms])
            tok = eng.next_token(ids, temperature=T, top_p=P, repetition_penalty=RP)
            toks.append(tok)
            logits.append(np.frombuffer(eng.last_logits(), np.float32).copy())
            for _ in range(len(uniforms) - 1):
                tok = eng.next_token(tok, temperature=T, top_p=P, repetition_penalty=RP)
                toks.append(tok)
                logits.append(np.frombuffer(eng.last_logits(), np.float32).copy())
        q_out.put((rank, "ok", toks, logits, eng.vocab_shard(), step_launches))
    except Exception as e:  # noqa: BLE001
        q_out.put((rank, "error", repr(e)[:400], None, None, None))


def _run_tp(wdir, shape, ids, teach, sampled=None, path=0):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, WORLD, wdir, shape.engine_kwargs(), ids, teach, q_id, q_out, sampled,
                                                        path))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in procs:
            r = q_out.get(timeout=600)
            out[r[0]] = r
    except queue.Empty:
        pass
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("shape_name,path", [("TINY", 0), ("TINY", 1), ("WIDE2", 0), ("WIDE2", 1)],
                         ids=["tiny-persistent", "tiny-per_op", "wide2-persistent", "wide2-per_op"])
def test_tp2_greedy_matches_oracle(built, shape_name, path):
    if _gpus() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    shape = getattr(S, shape_name)
    wdir = S.write_weight_tree(os.path.join("/tmp/xl_weights", shape_name.lower()), shape)
    port = O.Port(shape)
    port.load(wdir)
    ids = S.prompt_ids(3, 29, shape.vocab)
    steps = 10
    refs = [port.prefill(ids)]
    teach = []
    for _ in range(steps):
        teach.append(int(np.argmax(refs[-1])))
        refs.append(port.decode(teach[-1]))

    out = _run_tp(wdir, shape, ids, teach, path=path)
    assert sorted(out) == list(range(WORLD)), f"ranks missing: {out}"
    for r in range(WORLD):
        assert out[r][1] == "ok", out[r][2]
    if path == 0:
        # the persistent kernel (NVLink exchange of the split projections) + the greedy finish
        assert all(out[r][5] == 2 for r in range(WORLD)), [out[r][5] for r in range(WORLD)]
    shards = [out[r][4] for r in range(WORLD)]
    assert shards[0][0] == 0 and shards[-1][0] + shards[-1][1] == shape.vocab
    for r in range(1, WORLD):
        assert shards[r][0] == shards[r - 1][0] + shards[r - 1][1]
    for step, ref in enumerate(refs):
        got = np.concatenate([out[r][3][step] for r in range(WORLD)])
        span = float(ref.max() - ref.min())
        err = float(np.abs(got - ref).max())
        assert err <= 1e-3 * span, f"step {step}: max |dlogit| {err:.3e} > 1e-3 x {span:.3f}"
        toks = {out[r][2][step] for r in range(WORLD)}
        assert len(toks) == 1, f"step {step}: ranks disagree {toks}"
        tok, want = toks.pop(), int(np.argmax(ref))
        if tok != want:
            a = np.partition(ref, -2)[-2:]
            assert a[1] - a[0] < 1e-3 * span, f"step {step}: token {tok} != oracle {want}"


def _check_ranks(out, shape):
    assert sorted(out) == list(range(WORLD)), f"ranks missing: {out}"
    for r in range(WORLD):
        assert out[r][1] == "ok", out[r][2]
    shards = [out[r][4] for r in range(WORLD)]
    assert shards[0][0] == 0 and shards[-1][0] + shards[-1][1] == shape.vocab
    for r in range(1, WORLD):
        assert shards[r][0] == shards[r - 1][0] + shards[r - 1][1]


@pytest.mark.parametrize("shape_name,path", [("TINY", 0), ("WIDE2", 0), ("WIDE2", 1)],
                         ids=["tiny-persistent", "wide2-persistent", "wide2-per_op"])
def test_tp2_sampled_merge_matches_sample_cpu(built, shape_name, path):
    if _gpus() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    shape = getattr(S, shape_name)
    wdir = S.write_weight_tree(os.path.join("/tmp/xl_weights", shape_name.lower()), shape)
    T, P, RP = 0.7, 0.9, 1.1
    uniforms = S.philox_uniforms(3, 12)
    ids = S.prompt_ids(2, 41, shape.vocab)
    out = _run_tp(wdir, shape, ids, [], sampled=(T, P, RP, uniforms), path=path)
    _check_ranks(out, shape)
    port = O.Port(shape)
    port.load(wdir)
    history = []
    for step, r in enumerate(uniforms):
        toks = {out[q][2][step] for q in range(WORLD)}
        assert len(toks) == 1, f"step {step}: ranks disagree {toks}"
        tok = toks.pop()
        got = np.concatenate([out[q][3][step] for q in range(WORLD)])
        assert tok == O.sample(got, T, P, 1.0, [], float(r)), f"step {step}: merged draw differs from sample_cpu"
        ref = port.prefill(ids) if step == 0 else port.decode(out[0][2][step - 1])
        ref_pen = O.apply_penalty(ref, history, RP)
        span = float(ref_pen.max() - ref_pen.min())
        err = float(np.abs(got - ref_pen).max())
        assert err <= 1e-3 * span, f"step {step}: max |dlogit| {err:.3e} > 1e-3 x {span:.3f}"
        history.append(tok)
