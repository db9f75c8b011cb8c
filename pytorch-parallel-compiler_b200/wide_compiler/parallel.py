"""N-sharding of wide models across GPUs (one process per GPU).

The N fused models are independent, so the forward needs no communication:
each rank builds its wide model from a contiguous slice of the N models
(``shard_range`` / ``shard_models``) and runs it on its own GPU. The only
collective is the optional gather of every rank's output into the full
output at the unpack boundary, over NCCL on NVLink/NVSwitch (gloo on CPU for
tests):

* ``gather_outputs``: N-first outputs ``[n_local, ...]`` -> ``[N, ...]``.
  Even splits are one all-gather written straight into the result; ragged
  splits (N not a multiple of the world size) are one broadcast per rank,
  each written straight into that rank's rows of the result. No padding,
  no concatenation.
* ``gather_packed``: channel-packed outputs ``[B, n_local*F, ...]`` (what a
  TracedWideModel returns) -> ``[B, N*F, ...]``: the same collectives into a
  rank-major staging buffer, then one strided 2-D copy per rank places its
  rows (``widek_copy2d``).

``ShardedWideModel`` is the TracedWideModel path for several GPUs: this rank's
TracedWideModel over its slice of the models, which accepts either this
rank's packed input or the full packed input (its channel slice is cut out
on the device by one strided copy) and optionally gathers the full packed
output. The reference runs on one device only; nothing here has a reference
counterpart beyond the single-device pack/unpack boundary it slices
(wide_compiler/core/traced_wide.py:463-469, :527-532).
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn
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


def _group_ranks(group):
    """(this rank's index in the group, world size, global rank of each group index)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if group is None or group is dist.group.WORLD:
        globals_ = list(range(world))
    else:
        globals_ = [dist.get_global_rank(group, r) for r in range(world)]
    return rank, world, globals_


def gather_outputs(local: Tensor, n_total: int, group=None, out: Optional[Tensor] = None) -> Tensor:
    """All-gathers every rank's N-first output ``[n_local, ...]`` into
    ``[n_total, ...]`` on every rank (contiguous shards in rank order).
    ``out`` may supply the result buffer."""
    rank, world, globals_ = _group_ranks(group)
    a, b = shard_range(n_total, world, rank)
    if local.shape[0] != b - a:
        raise ValueError(f"rank {rank} holds {local.shape[0]} models, expected {b - a}")
    local = local.contiguous()
    if out is None:
        out = torch.empty((n_total, *local.shape[1:]), dtype=local.dtype, device=local.device)
    elif tuple(out.shape) != (n_total, *local.shape[1:]) or not out.is_contiguous():
        raise ValueError(f"gather_outputs: out must be a contiguous [{n_total}, {', '.join(map(str, local.shape[1:]))}]")
    if n_total % world == 0 and hasattr(dist, "all_gather_into_tensor") and dist.get_backend(group) != "gloo":
        dist.all_gather_into_tensor(out, local, group=group)
        return out
    # Ragged (or gloo): every rank broadcasts its rows straight into their
    # place in the result.
    out[a:b].copy_(local)
    for r in range(world):
        ra, rb = shard_range(n_total, world, r)
        if rb > ra:
            dist.broadcast(out[ra:rb], src=globals_[r], group=group)
    return out


def _start_gather_packed(local: Tensor, n_total: int, group=None):
    """Issues the collectives of ``gather_packed`` asynchronously and returns
    ``place(full)``, which waits for them (on the device: the current stream
    waits, the host does not block) and writes every rank's rows into the
    packed result ``full`` [B, n_total*F, *S] (one strided copy per rank)."""
    rank, world, globals_ = _group_ranks(group)
    a, b = shard_range(n_total, world, rank)
    n_local = b - a
    bsz = local.shape[0]
    if n_local == 0 or local.shape[1] % n_local:
        raise ValueError(f"gather_packed: {tuple(local.shape)} is not [B, {n_local}*F, ...]")
    f = local.shape[1] // n_local
    inner = f * math.prod(local.shape[2:])                 # elements per (sample, model)
    # One flat gather of every rank's [B, n_r, inner] block in rank order
    # (all-gather when the blocks are equal, else a broadcast per rank),
    # then one strided copy per rank into the packed result.
    blocks = [shard_range(n_total, world, r) for r in range(world)]
    sizes = [bsz * (rb - ra) * inner for ra, rb in blocks]
    offs = [0]
    for sz in sizes[:-1]:
        offs.append(offs[-1] + sz)
    flat = torch.empty(sum(sizes), dtype=local.dtype, device=local.device)
    mine = local.contiguous().reshape(-1)
    works = []
    if len(set(sizes)) == 1 and hasattr(dist, "all_gather_into_tensor") and dist.get_backend(group) != "gloo":
        works.append(dist.all_gather_into_tensor(flat, mine, group=group, async_op=True))
    else:
        flat[offs[rank]:offs[rank] + sizes[rank]].copy_(mine)
        for r in range(world):
            if sizes[r]:
                works.append(dist.broadcast(flat[offs[r]:offs[r] + sizes[r]], src=globals_[r], group=group,
                                            async_op=True))

    def place(full: Tensor) -> None:
        for w in works:
            w.wait()
        es = local.element_size()
        for r, (ra, rb) in enumerate(blocks):
            if rb == ra:
                continue
            row = (rb - ra) * inner * es
            copy_rows(flat[offs[r]:offs[r] + sizes[r]], row, full.view(bsz, n_total * inner)[:, ra * inner:],
                      n_total * inner * es, bsz, row)
    return place


def gather_packed(local: Tensor, n_total: int, group=None) -> Tensor:
    """All-gathers channel-packed outputs ``[B, n_local*F, *S]`` into
    ``[B, n_total*F, *S]`` on every rank (rank r's models at channels
    ``[lo_r*F, hi_r*F)``)."""
    place = _start_gather_packed(local, n_total, group)
    _, world, _ = _group_ranks(group)
    a, b = shard_range(n_total, world, _group_ranks(group)[0])
    f = local.shape[1] // (b - a)
    full = torch.empty((local.shape[0], n_total * f, *local.shape[2:]), dtype=local.dtype, device=local.device)
    place(full)
    return full


def copy_rows(src: Tensor, src_pitch: int, dst: Tensor, dst_pitch: int, rows: int, row_bytes: int) -> None:
    """``rows`` rows of ``row_bytes`` bytes from ``src`` (pitch ``src_pitch``
    bytes) into ``dst`` (pitch ``dst_pitch``), both starting at the views'
    first element: one libwidek strided-copy launch on CUDA tensors (a
    strided torch copy on CPU tensors, for the gloo tests)."""
    if rows == 0 or row_bytes == 0:
        return
    if src.is_cuda:
        from . import _native as N
        from .ops import _guard
        with _guard(dst.device):
            rc = N.lib().widek_copy2d(src.data_ptr(), src_pitch, dst.data_ptr(), dst_pitch, rows, row_bytes,
                                      N.stream_ptr(dst.device))
        N.check(rc, "widek_copy2d")
        return
    es = src.element_size()
    s = torch.as_strided(src, (rows, row_bytes // es), (src_pitch // es, 1))
    d = torch.as_strided(dst, (rows, row_bytes // es), (dst_pitch // es, 1))
    d.copy_(s)


class ShardedWideModel(nn.Module):
    """This rank's share of a wide model fused from N models.

    Builds a TracedWideModel (``compile_model=True``: the CUDA-graph executor
    around it) from this rank's contiguous slice of ``models``
    (``shard_range``). ``forward(x)`` takes either this rank's packed input
    ``[B, n_local*C, ...]`` or the full packed input ``[B, N*C, ...]``, whose
    channel slice ``[lo*C, hi*C)`` is cut out on the device by one strided
    copy; it returns this rank's packed output ``[B, n_local*F, ...]`` or,
    with ``gather=True``, the full packed output ``[B, N*F, ...]`` on every
    rank (``gather_packed``: the only collective).

    ``gather_chunks=k`` (> 1) overlaps that gather with the forward: the
    batch runs as k consecutive slices (contiguous in the packed layout, so
    no copy), each slice's gather is issued asynchronously as soon as its
    forward has been queued, and runs on NCCL's stream while the next slice
    computes; the rows land in the result after the last forward. Used only
    when the result cannot depend on the batch split: no BatchNorm in
    training mode.
    """

    def __init__(self, models: Sequence[nn.Module], sample_input: Tensor, rank: Optional[int] = None,
                 world: Optional[int] = None, group=None, gather: bool = False, compile_model: bool = False,
                 gather_chunks: int = 1):
        super().__init__()
        if gather_chunks < 1:
            raise ValueError(f"gather_chunks must be >= 1, got {gather_chunks}")
        self.gather_chunks = gather_chunks
        from .api import compile as wide_compile
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        self.n_total = len(models)
        self.lo, self.hi = shard_range(self.n_total, self.world, self.rank)
        if self.hi <= self.lo:
            raise ValueError(f"rank {self.rank} owns no models (N={self.n_total}, world={self.world})")
        self.gather = gather
        self.channels = sample_input.shape[1]          # C of one model's input [B, C, ...]
        self.local = wide_compile(list(models[self.lo:self.hi]), sample_input, compile_model=compile_model,
                                  debug=False)

    @property
    def n_local(self) -> int:
        return self.hi - self.lo

    def local_input(self, x: Tensor) -> Tensor:
        """This rank's packed input: ``x`` itself when it holds n_local*C
        channels, its channel slice [lo*C, hi*C) when it holds N*C."""
        c = self.channels
        if x.shape[1] == self.n_local * c:
            return x
        if x.shape[1] != self.n_total * c:
            raise ValueError(f"ShardedWideModel: input dim 1 is {x.shape[1]}, expected {self.n_local}*{c} "
                             f"(this rank's models) or {self.n_total}*{c} (all models)")
        xs = x if x.is_contiguous() else x.contiguous()
        inner = c * math.prod(x.shape[2:])
        out = torch.empty((x.shape[0], self.n_local * c, *x.shape[2:]), dtype=x.dtype, device=x.device)
        es = x.element_size()
        copy_rows(xs.view(x.shape[0], -1)[:, self.lo * inner:], self.n_total * inner * es, out,
                  self.n_local * inner * es, x.shape[0], self.n_local * inner * es)
        return out

    def _batch_split_ok(self) -> bool:
        return not any(isinstance(m, nn.modules.batchnorm._BatchNorm) and m.training for m in self.local.modules())

    def forward(self, x: Tensor) -> Tensor:
        xl = self.local_input(x)
        if not (self.gather and self.world > 1):
            return self.local(xl)
        k = min(self.gather_chunks, xl.shape[0])
        if k <= 1 or not self._batch_split_ok():
            return gather_packed(self.local(xl), self.n_total, group=self.group)
        places, full = [], None
        for c in range(k):
            b0, b1 = shard_range(xl.shape[0], k, c)
            y = self.local(xl[b0:b1])
            if full is None:
                f = y.shape[1] // self.n_local
                full = torch.empty((xl.shape[0], self.n_total * f, *y.shape[2:]), dtype=y.dtype, device=y.device)
            places.append((b0, b1, _start_gather_packed(y, self.n_total, self.group)))
        for b0, b1, place in places:
            place(full[b0:b1])
        return full


__all__ = ['shard_range', 'shard_models', 'gather_outputs', 'gather_packed', 'copy_rows', 'ShardedWideModel']
