"""Packing between N per-model tensors and the channel-packed wide layout.

pack_inputs:    N x [B, F, *S]  ->  [B, N*F, *S]
unpack_outputs: [B, N*F, *S]    ->  N x [B, F, *S] (views)

Same contract and errors as the reference
(wide_compiler/core/ensemble_util.py:20-101). On CUDA the stack is one
libwidek kernel over the N source pointers; other devices are rejected by
the kernel wrapper (there is no host implementation of the wide path).
"""
from __future__ import annotations

from typing import List

from torch import Tensor


def pack_inputs(inputs: List[Tensor]) -> Tensor:
    """Stacks N inputs [B, F, *S] along a new dim 1 and flattens it into F."""
    if not inputs:
        raise ValueError("inputs list is empty")
    from .. import ops
    stacked = ops.pack(list(inputs))            # [B, N, *F]
    b, n = stacked.shape[0], stacked.shape[1]
    rest = stacked.shape[2:]
    if len(rest) == 0:
        return stacked.view(b, n)
    return stacked.view(b, n * rest[0], *rest[1:])


def unpack_outputs(output: Tensor, n: int) -> List[Tensor]:
    """Splits dim 1 of [B, N*F, *S] into N views [B, F, *S]."""
    if output.dim() < 2:
        raise ValueError("output must have at least 2 dimensions")
    b, nf = output.shape[0], output.shape[1]
    if nf % n != 0:
        raise ValueError(f"Cannot split dim 1 ({nf}) into {n} equal parts")
    v = output.view(b, n, nf // n, *output.shape[2:])
    return [v[:, i] for i in range(n)]


__all__ = ['pack_inputs', 'unpack_outputs']
