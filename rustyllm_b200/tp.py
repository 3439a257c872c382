"""Tensor-parallel plumbing: one process per GPU, the NCCL id from rank 0
handed to every rank over torch.distributed, and the sharding rule of the
Llama linears (column-parallel q/k/v/gate/up and lm_head, row-parallel
o/down)."""
from __future__ import annotations

import ctypes

from . import _lib
from ._lib import check

ID_BYTES = 128


def init_from_torch(ctx, timeout_ms: int = 60000) -> tuple[int, int]:
    """rq_tp_init on ctx for the current torch.distributed group."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(), dist.get_rank()
    obj = [None]
    if rank == 0:
        buf = ctypes.create_string_buffer(ID_BYTES)
        check(_lib.lib().rq_tp_unique_id(buf, ID_BYTES))
        obj = [buf.raw]
    dist.broadcast_object_list(obj, src=0)
    uid = ctypes.create_string_buffer(obj[0], ID_BYTES)
    check(_lib.lib().rq_tp_init(ctx.handle, world, rank, uid, timeout_ms))
    return world, rank


def world_rank(ctx=None) -> tuple[int, int]:
    """(world, rank) of the current torch.distributed group, (1, 0) without
    one; the context's communicator (init_from_torch) spans that group."""
    try:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            return dist.get_world_size(), dist.get_rank()
    except Exception:
        pass
    return 1, 0


def finalize(ctx) -> None:
    _lib.lib().rq_tp_finalize(ctx.handle)


def shard(kind: str, t, world: int, rank: int):
    """Rank's shard of a full [out, in] matrix: rows for column-parallel
    ("col": q, k, v, gate, up, lm_head), columns for row-parallel ("row": o,
    down).  Splits fall on 256-element super-block boundaries for the sizes
    rq_llama_create accepts, so quantizing a shard gives exactly the blocks
    of the full matrix."""
    if world == 1:
        return t
    if kind == "col":
        n = t.shape[0] // world
        return t[rank * n:(rank + 1) * n]
    n = t.shape[1] // world
    return t[:, rank * n:(rank + 1) * n].contiguous()


# q, k, v, o, gate, up, down
LINEAR_SPLIT = ("col", "col", "col", "row", "col", "col", "row")
