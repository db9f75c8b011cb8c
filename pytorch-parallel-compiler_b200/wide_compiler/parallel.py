"""N-sharding of wide models across GPUs (one process per GPU).

The N fused models are independent, so the forward needs no communication:
each rank builds its wide model from a contiguous slice of the N models
(``shard_range`` / ``shard_models``) and runs it on its own GPU. The only
collective is the optional gather of every rank's N-first output into the
full ``[N, ...]`` tensor at the unpack boundary (``gather_outputs``), over
NCCL on NVLink/NVSwitch (gloo on CPU for tests). Ragged splits (N not a
multiple of the world size) are padded to ceil(N / world) rows per rank for
the collective and trimmed afterwards.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
from torch import Tensor


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of the models owned by ``rank``: contiguous slices, the
    first ``n % world`` ranks get one extra model (e.g. N=100 on 8 GPUs:
    13,13,13,13,12,12,12,12)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_models(models: Sequence, rank: Optional[int] = None, world: Optional[int] = None) -> List:
    """The sub-list of ``models`` this rank builds its wide model from."""
    rank = dist.get_rank() if rank is None else rank
    world = dist.get_world_size() if world is None else world
    a, b = shard_range(len(models), world, rank)
    return list(models[a:b])


def gather_outputs(local: Tensor, n_total: int, group=None) -> Tensor:
    """All-gathers every rank's N-first output [n_local, ...] into
    [n_total, ...] on every rank (contiguous shards in rank order)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    per = -(-n_total // world)
    a, b = shard_range(n_total, world, rank)
    if local.shape[0] != b - a:
        raise ValueError(f"rank {rank} holds {local.shape[0]} models, expected {b - a}")
    padded = local
    if local.shape[0] != per:
        padded = torch.zeros((per, *local.shape[1:]), dtype=local.dtype, device=local.device)
        padded[:local.shape[0]] = local
    padded = padded.contiguous()
    if local.is_cuda and hasattr(dist, "all_gather_into_tensor"):
        full = torch.empty((per * world, *local.shape[1:]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(full, padded, group=group)
        parts = [full[r * per:(r + 1) * per] for r in range(world)]
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded, group=group)
    out = []
    for r in range(world):
        ra, rb = shard_range(n_total, world, r)
        out.append(parts[r][:rb - ra])
    return torch.cat(out, dim=0)


__all__ = ['shard_range', 'shard_models', 'gather_outputs']
