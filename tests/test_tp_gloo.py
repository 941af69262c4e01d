"""Host logic of tensor-parallel decode on CPU: two gloo ranks (world size 2)
exchange the NCCL id and their shard plans exactly as the GPU path does, and a
rank that fails before a collective surfaces as an error on its peer (no hang).
No GPU, no NCCL communicator: the failure is made on the host."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    sys.path[:0] = [os.path.join(ROOT, "xingling-cpp_b200")]
    from datetime import timedelta

    import torch.distributed as dist

    import xl_tp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the exchange")
        ident = xl_tp.share_nccl_id(dist, rank, make_id=lambda: bytes(range(128)))
        plan = xl_tp.tp_plan(world, rank)
        plans = [None] * world
        dist.all_gather_object(plans, plan)
        q.put((rank, "ok", ident == bytes(range(128)), plans))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", type(e).__name__, str(e)[:200]))
    finally:
        if mode != "fail":
            dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out)


def test_tp_bootstrap_two_ranks(built):
    res = _run("ok")
    assert [r[1] for r in res] == ["ok", "ok"]
    assert all(r[2] for r in res)  # both ranks hold rank 0's id
    plans = res[0][3]
    assert plans == res[1][3]
    assert [p["heads"] for p in plans] == [12, 12]
    assert [p["ffn"] for p in plans] == [2048, 2048]
    assert plans[0]["vocab_begin"] == 0 and plans[1]["vocab_begin"] == plans[0]["vocab_count"]
    assert plans[0]["vocab_count"] + plans[1]["vocab_count"] == 151669


def test_tp_rank_failure_surfaces_as_error(built):
    res = _run("fail")
    by_rank = {r[0]: r for r in res}
    assert by_rank[1][1] == "error"
    assert by_rank[0][1] == "error"  # the peer's collective ends with an error, within the group timeout
