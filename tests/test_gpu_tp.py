"""Tensor-parallel decode on 2, 4 and 8 GPUs (each case skipped when fewer are
visible): spawned ranks, each one shard of the engine on its own GPU with the
engine's own NCCL communicator (rank 0's id handed over through a queue),
against the oracle port on the same weight tree.

Both decode paths: the persistent kernel (the out-projection and W2 partial
sums of every CTA go, tagged, to every rank's exchange buffer over NVLink and
each rank sums them in the same order; the ranks' argmax keys merge there
too, so a greedy step is this one kernel) and the per-op path (NCCL
all-reduces).  The shard widths covered: heads
12/6/3 per rank, attention widths 768/384/192 (k-tiles of 256/128/64 in the
persistent kernel's weight boxes), FFN columns 2048/1024/512, contiguous
vocab shards.

* Greedy, teacher-forced on the oracle's ids: the ranks' vocab shards,
  concatenated, match the oracle's logits within 1e-3 of their range, and
  every rank returns the same id (the greedy merge of per-shard maxima).
* XingLing-0.68B itself (prompt of 64 ids, seed 4, 256 greedy steps): the
  tensor-parallel decode workload, at every width.
* Sampled (temperature 0.7, top_p 0.9, repetition penalty 1.1, the same
  Philox uniforms queued on both ranks), free-running: every rank returns the
  same id, which is exactly sample_cpu's draw on the concatenated penalised
  logits (the all-gather merge of per-shard top-1024 lists), and those logits
  match the oracle's, penalised with the engine's own history, within 1e-3 of
  their range.
* Greedy generate on the device (every rank the same call): the same ids as
  the next_token loop, one generation-graph launch per step.
* A rank that stops calling between steps: the survivor's next step ends
  with RuntimeError within its step timeout (the communicator is aborted, no
  GPU work is left waiting), and the engine refuses later steps.

NVLS stays off: a rank that fails must not leave memory bound to an NVLink
multicast object."""
import os
import queue
import sys
import tempfile
import time

import numpy as np
import pytest

import oracle as O
import xl_synth as S

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _need(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")


def _engine(rank, world, shape_kw, q_id, path):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path[:0] = [os.path.join(ROOT, "xingling-cpp_b200")]
    import llm_cpp_engine as m

    if rank == 0:
        ident = m.nccl_unique_id()
        for _ in range(world - 1):
            q_id.put(ident)
    else:
        ident = q_id.get(timeout=120)
    eng = m.InferenceEngine(f"cuda:{rank}", tp=world, rank=rank, nccl_id=ident, **shape_kw)
    eng.set_option("decode_path", path)
    return m, eng


def _rank(rank, world, wdir, shape_kw, ids, teach, q_id, q_out, sampled=None, path=0, out_dir=None):
    """One rank: prefill + decode steps; its per-step ids and logits shard go
    back through q_out (or, with out_dir, into an .npy file there)."""
    try:
        m, eng = _engine(rank, world, shape_kw, q_id, path)
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
        if out_dir is not None:
            fn = os.path.join(out_dir, f"logits_{rank}.npy")
            np.save(fn, np.stack(logits))
            logits = fn
        q_out.put((rank, "ok", toks, logits, eng.vocab_shard(), step_launches))
    except Exception as e:  # noqa: BLE001
        q_out.put((rank, "error", repr(e)[:400], None, None, None))


def _spawn(world, target, args_of, timeout=300):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=target, args=args_of(r, q_id, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in procs:
            r = q_out.get(timeout=timeout)
            out[r[0]] = r
    except queue.Empty:
        pass
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def _run_tp(world, wdir, shape, ids, teach, sampled=None, path=0, out_dir=None):
    return _spawn(world, _rank, lambda r, q_id, q_out: (r, world, wdir, shape.engine_kwargs(), ids, teach, q_id,
                                                         q_out, sampled, path, out_dir))


def _check_ranks(out, shape, world):
    assert sorted(out) == list(range(world)), f"ranks missing: {out}"
    for r in range(world):
        assert out[r][1] == "ok", out[r][2]
    shards = [out[r][4] for r in range(world)]
    assert shards[0][0] == 0 and shards[-1][0] + shards[-1][1] == shape.vocab
    for r in range(1, world):
        assert shards[r][0] == shards[r - 1][0] + shards[r - 1][1]


def _rank_logits(out, world):
    per = [out[r][3] for r in range(world)]
    return [np.load(x) if isinstance(x, str) else np.stack(x) for x in per]


def _check_greedy(out, refs, shape, world, path):
    _check_ranks(out, shape, world)
    if path == 0:
        # the persistent kernel alone: the split projections' partial sums and the greedy merge of the
        # ranks' argmax keys cross NVLink inside it
        assert all(out[r][5] == 1 for r in range(world)), [out[r][5] for r in range(world)]
    shards = _rank_logits(out, world)
    for step, ref in enumerate(refs):
        got = np.concatenate([shards[r][step] for r in range(world)])
        span = float(ref.max() - ref.min())
        err = float(np.abs(got - ref).max())
        assert err <= 1e-3 * span, f"step {step}: max |dlogit| {err:.3e} > 1e-3 x {span:.3f}"
        toks = {out[r][2][step] for r in range(world)}
        assert len(toks) == 1, f"step {step}: ranks disagree {toks}"
        tok, want = toks.pop(), int(np.argmax(ref))
        if tok != want:
            a = np.partition(ref, -2)[-2:]
            assert a[1] - a[0] < 1e-3 * span, f"step {step}: token {tok} != oracle {want}"


def _oracle_greedy(port, ids, steps):
    refs = [port.prefill(ids)]
    teach = []
    for _ in range(steps):
        teach.append(int(np.argmax(refs[-1])))
        refs.append(port.decode(teach[-1]))
    return refs, teach


SMALL = [("TINY", 2, 0), ("TINY", 2, 1), ("TINY", 4, 0), ("WIDE2", 2, 0), ("WIDE2", 2, 1), ("WIDE2", 4, 0),
         ("WIDE2", 4, 1), ("WIDE2", 8, 0), ("WIDE2", 8, 1)]


@pytest.mark.parametrize("shape_name,world,path", SMALL,
                         ids=[f"{s.lower()}-tp{w}-{'persistent' if p == 0 else 'per_op'}" for s, w, p in SMALL])
def test_tp_greedy_matches_oracle(built, shape_name, world, path):
    _need(world)
    shape = getattr(S, shape_name)
    wdir = S.write_weight_tree(os.path.join("/tmp/xl_weights", shape_name.lower()), shape)
    port = O.Port(shape)
    port.load(wdir)
    ids = S.prompt_ids(3, 29, shape.vocab)
    refs, teach = _oracle_greedy(port, ids, 10)
    out = _run_tp(world, wdir, shape, ids, teach, path=path)
    _check_greedy(out, refs, shape, world, path)


FULL_CASES = [(2, 0, 256), (2, 1, 32), (4, 0, 256), (4, 1, 32), (8, 0, 256), (8, 1, 32)]


@pytest.mark.parametrize("world,path,steps", FULL_CASES,
                         ids=[f"tp{w}-{'persistent' if p == 0 else 'per_op'}" for w, p, _ in FULL_CASES])
def test_tp_full_model_greedy_matches_oracle(built, full_weights, world, path, steps):
    """XingLing-0.68B, prompt of 64 ids (seed 4), greedy decode teacher-forced
    on the oracle: 256 steps on the persistent kernel (the whole workload),
    32 on the per-op path."""
    _need(world)
    shape = S.FULL
    port = O.Port(shape)
    port.load(full_weights)
    ids = S.prompt_ids(4, 64, shape.vocab)
    refs, teach = _oracle_greedy(port, ids, steps)
    with tempfile.TemporaryDirectory(prefix="xl_tp_") as d:
        out = _run_tp(world, full_weights, shape, ids, teach, path=path, out_dir=d)
        _check_greedy(out, refs, shape, world, path)


SAMPLED = [("TINY", 2, 0), ("WIDE2", 2, 0), ("WIDE2", 2, 1), ("WIDE2", 8, 0)]


@pytest.mark.parametrize("shape_name,world,path", SAMPLED,
                         ids=[f"{s.lower()}-tp{w}-{'persistent' if p == 0 else 'per_op'}" for s, w, p in SAMPLED])
def test_tp_sampled_merge_matches_sample_cpu(built, shape_name, world, path):
    _need(world)
    shape = getattr(S, shape_name)
    wdir = S.write_weight_tree(os.path.join("/tmp/xl_weights", shape_name.lower()), shape)
    T, P, RP = 0.7, 0.9, 1.1
    uniforms = S.philox_uniforms(3, 12)
    ids = S.prompt_ids(2, 41, shape.vocab)
    out = _run_tp(world, wdir, shape, ids, [], sampled=(T, P, RP, uniforms), path=path)
    _check_ranks(out, shape, world)
    shards = _rank_logits(out, world)
    port = O.Port(shape)
    port.load(wdir)
    history = []
    for step, r in enumerate(uniforms):
        toks = {out[q][2][step] for q in range(world)}
        assert len(toks) == 1, f"step {step}: ranks disagree {toks}"
        tok = toks.pop()
        got = np.concatenate([shards[q][step] for q in range(world)])
        assert tok == O.sample(got, T, P, 1.0, [], float(r)), f"step {step}: merged draw differs from sample_cpu"
        ref = port.prefill(ids) if step == 0 else port.decode(out[0][2][step - 1])
        ref_pen = O.apply_penalty(ref, history, RP)
        span = float(ref_pen.max() - ref_pen.min())
        err = float(np.abs(got - ref_pen).max())
        assert err <= 1e-3 * span, f"step {step}: max |dlogit| {err:.3e} > 1e-3 x {span:.3f}"
        history.append(tok)


def _rank_stops(rank, world, wdir, shape_kw, ids, q_id, q_out, q_ctl, path, timeout_ms):
    """Both ranks prefill and decode two steps.  Then rank 1 stops calling (its
    host is stuck; nothing of it is in flight) until the test releases it;
    rank 0 takes one more step, which must end in RuntimeError within its step
    timeout, then a refused step, then destroys its engine."""
    import faulthandler

    faulthandler.dump_traceback_later(150, exit=False)  # a stuck call shows up in the log
    os.environ["XL_TRACE_ABORT"] = "1"
    try:
        m, eng = _engine(rank, world, shape_kw, q_id, path)
        eng.load(wdir)
        tok = eng.next_token(ids, top_p=0.0, repetition_penalty=1.0)
        for _ in range(2):
            tok = eng.next_token(tok, top_p=0.0, repetition_penalty=1.0)
        if rank != 0:
            q_out.put((rank, "stopped", tok, None, None, None))
            q_ctl.get(timeout=300)  # released once rank 0 has reported
            os._exit(0)  # leaves without a collective: the communicator's peer is gone
        eng.set_option("step_timeout_ms", timeout_ms)
        print("[rank 0] stepping without the peer", file=sys.stderr, flush=True)
        t0 = time.monotonic()
        try:
            eng.next_token(tok, top_p=0.0, repetition_penalty=1.0)
            first = ("no error", time.monotonic() - t0)
        except RuntimeError as e:
            first = (str(e)[:300], time.monotonic() - t0)
        t1 = time.monotonic()
        try:
            eng.next_token(tok, top_p=0.0, repetition_penalty=1.0)
            second = ("no error", time.monotonic() - t1)
        except RuntimeError as e:
            second = (str(e)[:300], time.monotonic() - t1)
        print(f"[rank 0] first {first}, second {second}", file=sys.stderr, flush=True)
        t2 = time.monotonic()
        del eng
        print("[rank 0] engine destroyed", file=sys.stderr, flush=True)
        q_out.put((rank, "ok", first, second, time.monotonic() - t2, None))
    except Exception as e:  # noqa: BLE001
        q_out.put((rank, "error", repr(e)[:400], None, None, None))


def _rank_generate(rank, world, wdir, shape_kw, ids, steps, q_id, q_out):
    """One rank: greedy generate(steps) after a prefill, then the same steps as
    a next_token loop after the same prefill again; both id lists, the
    positions and the launches the generate call made."""
    try:
        m, eng = _engine(rank, world, shape_kw, q_id, 0)
        eng.load(wdir)
        tok = eng.next_token(ids, top_p=0.0, repetition_penalty=1.0)
        n0 = m.kernel_launches()
        gen = eng.generate(tok, steps, top_p=0.0, repetition_penalty=1.0)
        launches = m.kernel_launches() - n0
        ctx_gen = eng.ctx_len()
        tok2 = eng.next_token(ids, top_p=0.0, repetition_penalty=1.0)
        loop, t = [], tok2
        for _ in range(steps):
            t = eng.next_token(t, top_p=0.0, repetition_penalty=1.0)
            loop.append(t)
        q_out.put((rank, "ok", gen, loop, (tok, tok2, ctx_gen, eng.ctx_len()), launches))
    except Exception as e:  # noqa: BLE001
        q_out.put((rank, "error", repr(e)[:400], None, None, None))


GEN_WORLDS = [2, 4, 8]


@pytest.mark.parametrize("world", GEN_WORLDS, ids=[f"wide2-tp{w}" for w in GEN_WORLDS])
def test_tp_generate_on_device_matches_next_token_loop(built, world):
    """Greedy generate on tensor-parallel engines runs on the device: one
    launch of the generation graph per step on every rank (gen_feed, the
    persistent kernel after the step-start all-reduce, gen_collect), no host
    round trip between steps, and the same ids, on every rank, as the
    next_token loop after the same prefill."""
    _need(world)
    shape = S.WIDE2
    wdir = S.write_weight_tree(os.path.join("/tmp/xl_weights", "wide2"), shape)
    ids = S.prompt_ids(7, 31, shape.vocab)
    steps = 40
    out = _spawn(world, _rank_generate,
                 lambda r, q_id, q_out: (r, world, wdir, shape.engine_kwargs(), ids, steps, q_id, q_out))
    assert sorted(out) == list(range(world)), f"ranks missing: {out}"
    for r in range(world):
        assert out[r][1] == "ok", out[r][2]
    for r in range(world):
        tok, tok2, ctx_gen, ctx_loop = out[r][4]
        assert tok == tok2
        assert out[r][2] == out[r][3], f"rank {r}: generate {out[r][2]} != loop {out[r][3]}"
        assert out[r][2] == out[0][2], "ranks disagree"
        assert ctx_gen == ctx_loop == len(ids) + steps
        assert out[r][5] == 3 * steps, f"rank {r}: {out[r][5]} launches for {steps} steps"


@pytest.mark.parametrize("path", [0, 1], ids=["persistent", "per_op"])
def test_tp_peer_stops_survivor_raises_within_timeout(built, tiny_weights, path):
    _need(2)
    import torch.multiprocessing as mp

    shape = S.TINY
    timeout_ms = 2000
    ctx = mp.get_context("spawn")
    q_id, q_out, q_ctl = ctx.Queue(), ctx.Queue(), ctx.Queue()
    ids = S.prompt_ids(3, 29, shape.vocab)
    procs = [ctx.Process(target=_rank_stops, args=(r, 2, tiny_weights, shape.engine_kwargs(), ids, q_id, q_out, q_ctl,
                                                     path, timeout_ms)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in procs:
            r = q_out.get(timeout=240)
            out[r[0]] = r
    except queue.Empty:
        pass
    finally:
        q_ctl.put("done")
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert sorted(out) == [0, 1], f"ranks missing: {out}"
    assert out[1][1] == "stopped", out[1]
    assert out[0][1] == "ok", out[0][2]
    (msg1, dt1), (msg2, dt2), dt_del = out[0][2], out[0][3], out[0][4]
    assert "did not finish within" in msg1 and "aborted" in msg1, msg1
    assert timeout_ms / 1000 <= dt1 < timeout_ms / 1000 + 15, f"first failing step took {dt1:.1f} s"
    assert "unusable" in msg2 and dt2 < 1.0, (msg2, dt2)
    assert dt_del < 30, f"destroying the aborted engine took {dt_del:.1f} s"
