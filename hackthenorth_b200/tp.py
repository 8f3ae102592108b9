"""Tensor-parallel group setup over torch.distributed (one process per GPU).

The decode kernels run their own NCCL communicator (inside libqb.so) so the
all-reduces can live in the captured decode graph; torch.distributed only
carries the NCCL unique id from rank 0 to the others.
"""
from __future__ import annotations

import torch

from . import _lib


def unique_id() -> bytes:
    """A fresh NCCL unique id (call on rank 0)."""
    buf = _lib.ctypes.create_string_buffer(128)
    _lib.check(_lib.load().qb_nccl_unique_id(buf, 128))
    return buf.raw


def shared_unique_id() -> bytes:
    """Rank 0 creates the id and broadcasts it through the default process group."""
    import torch.distributed as dist

    obj = [unique_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def engine_from_random(cfg, seed: int = 0, init_device=None):
    """Build this rank's tensor-parallel Engine (weights drawn on its GPU, same
    seed on every rank, so the shards come from one model)."""
    import torch.distributed as dist

    from .engine import Engine

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = f"cuda:{torch.cuda.current_device()}"
    uid = shared_unique_id() if world > 1 else None
    return Engine.from_random(cfg, seed, device=dev, init_device=init_device or dev, tp_rank=rank,
                              tp_size=world, unique_id=uid)
