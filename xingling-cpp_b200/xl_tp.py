"""Tensor-parallel bootstrap for llm_cpp_engine on one node.

One process per GPU.  Rank 0 creates the NCCL unique id (128 bytes) through
the engine library, every rank receives it over the caller's
torch.distributed process group, then each rank builds its engine shard:
heads, FFN columns and a contiguous vocab shard (see xl_tp_plan in
include/xl_engine.h).  Every rank must then call next_token with the same
arguments in the same order; ranks agree on every sampled id (greedy merge of
(value, id) maxima across vocab shards).
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "libxl_engine.so")


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("layers", "hidden", "heads", "ffn", "vocab", "max_ctx")] + \
               [("rope_base", C.c_float)]


def tp_plan(tp: int, rank: int, layers=16, hidden=1536, heads=24, ffn=4096, vocab=151669, max_ctx=768) -> dict:
    """This rank's shard: heads, attention width, FFN columns, vocab range."""
    lib = C.CDLL(_LIB)
    cfg = _Cfg(layers, hidden, heads, ffn, vocab, max_ctx, 10000.0)
    out = (C.c_int * 5)()
    if lib.xl_tp_plan(C.byref(cfg), tp, rank, out) != 0:
        lib.xl_last_error.restype = C.c_char_p
        raise ValueError(lib.xl_last_error().decode())
    return {"heads": out[0], "hidden": out[1], "ffn": out[2], "vocab_begin": out[3], "vocab_count": out[4]}


def share_nccl_id(dist, rank: int, make_id=None) -> bytes:
    """Rank 0's NCCL unique id, broadcast to every rank of the default group."""
    if make_id is None:
        import llm_cpp_engine

        make_id = llm_cpp_engine.nccl_unique_id
    holder = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(holder, src=0)
    ident = holder[0]
    if not isinstance(ident, (bytes, bytearray)) or len(ident) != 128:
        raise RuntimeError("tensor parallel: malformed NCCL id from rank 0")
    return bytes(ident)


def make_tp_engine(dist, rank: int, world: int, local_rank: int, **shape):
    """Create this rank's shard of a tensor-parallel engine (all ranks call together)."""
    import llm_cpp_engine

    ident = share_nccl_id(dist, rank)
    return llm_cpp_engine.InferenceEngine(f"cuda:{local_rank}", tp=world, rank=rank, nccl_id=ident, **shape)
