"""Tensor-parallel decode on two GPUs (skipped with fewer): two spawned ranks,
each one shard of the engine on its own GPU with the engine's own NCCL
communicator (rank 0's id handed over through a queue), against the oracle
port on the same weight tree.  Greedy and teacher-forced on the oracle's ids;
the ranks' vocab shards, concatenated, must match the oracle's logits within
1e-3 of their range, and every rank must return the same id (the greedy merge
of per-shard (value, id) maxima).  NVLS stays off: a rank that fails must not
leave memory bound to an NVLink multicast object."""
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


def _rank(rank, world, wdir, shape_kw, ids, teach, q_id, q_out):
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
        eng.load(wdir)
        toks, logits = [], []
        tok = eng.next_token(ids, top_p=0.0, repetition_penalty=1.0)
        toks.append(tok)
        logits.append(np.frombuffer(eng.last_logits(), np.float32).copy())
        for t in teach:
            tok = eng.next_token(int(t), top_p=0.0, repetition_penalty=1.0)
            toks.append(tok)
            logits.append(np.frombuffer(eng.last_logits(), np.float32).copy())
        q_out.put((rank, "ok", toks, logits, eng.vocab_shard()))
    except Exception as e:  # noqa: BLE001
        q_out.put((rank, "error", repr(e)[:400], None, None))


def _run_tp(wdir, shape, ids, teach):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, WORLD, wdir, shape.engine_kwargs(), ids, teach, q_id, q_out))
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


@pytest.mark.parametrize("shape_name", ["TINY", "WIDE2"])
def test_tp2_greedy_matches_oracle(built, shape_name):
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

    out = _run_tp(wdir, shape, ids, teach)
    assert sorted(out) == list(range(WORLD)), f"ranks missing: {out}"
    for r in range(WORLD):
        assert out[r][1] == "ok", out[r][2]
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
