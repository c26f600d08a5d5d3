"""Data-parallel sharding of the policy forward across ranks (one GPU each).

States are independent, so a global batch of world * B states splits into
contiguous shards with no collective on the data path. The only exchange is
the weight broadcast from rank 0. On GPUs the library does it: one
ncclBroadcast of the packed device weight arena (EncoderPolicy.broadcast_from),
over a communicator whose 128-byte id travels through torch.distributed
(share_comm_id). broadcast_weights moves the f32 blob itself, for CPU ranks
(gloo) and tests.
"""
from __future__ import annotations

import numpy as np

from .presets import PolicyConfig
from .synth import make_inputs, make_weights


def shard_range(rank: int, per_rank: int) -> tuple[int, int]:
    """Global state indices [lo, hi) owned by `rank` when each rank holds `per_rank` states."""
    return rank * per_rank, (rank + 1) * per_rank


def shard_inputs(cfg: PolicyConfig, seed: int, rank: int, per_rank: int | None = None):
    """This rank's features/counts: the global states of its shard, bit-identical
    to the same states of an unsharded batch."""
    B = cfg.batch if per_rank is None else int(per_rank)
    lo, _ = shard_range(rank, B)
    return make_inputs(cfg, batch=B, seed=seed, state_offset=lo)


def broadcast_weights(cfg: PolicyConfig, seed: int, rank: int, device=None) -> np.ndarray:
    """Rank 0 builds the seeded weight blob; one broadcast gives every rank the
    same blob (torch.distributed must be initialised; `device` is the rank's GPU
    for NCCL or None/'cpu' for gloo)."""
    import torch
    import torch.distributed as dist

    from .synth import weight_count

    n = weight_count(cfg)
    t = torch.empty(n, dtype=torch.float32, device=device if device is not None else "cpu")
    if rank == 0:
        t.copy_(torch.from_numpy(make_weights(cfg, seed=seed)))
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.broadcast(t, src=0)
    return t.cpu().numpy()


def share_comm_id(rank: int, uid: bytes | None = None) -> bytes:
    """The NCCL id (ow_comm_unique_id on rank 0) handed to every rank over the
    initialised torch.distributed group: host plumbing only, 128 bytes once."""
    import torch.distributed as dist

    obj = [uid if rank == 0 else None]
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.broadcast_object_list(obj, src=0)
    if obj[0] is None or len(obj[0]) != 128:
        raise RuntimeError("communicator id did not arrive")
    return obj[0]
