"""WideLayerNorm: N LayerNorms over the last dim, one single-pass kernel.

Parameter layout as the reference (wide_layernorm.py:38-39): flat
``weight``/``bias`` of N*D. Forward [N, B, ..., D] -> same shape with biased
variance and the module's eps (reference :41-67). Statistics are computed in
fp32 inside the kernel for every storage dtype.
"""
from __future__ import annotations

from typing import List

import torch
from torch import Tensor, nn

from ... import ops


class WideLayerNorm(nn.Module):
    """N parallel LayerNorm(D) with per-model affine."""

    def __init__(self, n: int, normalized_shape: int, eps: float = 1e-5):
        super().__init__()
        self.n = n
        self.normalized_shape = normalized_shape
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(n * normalized_shape))
        self.bias = nn.Parameter(torch.zeros(n * normalized_shape))

    def forward(self, x: Tensor) -> Tensor:
        return ops.layernorm(x, self.weight, self.bias, self.n, self.normalized_shape, self.eps)

    def forward_packed(self, x: Tensor) -> Tensor:
        """The same LayerNorm on the packed boundary layout [B, N*T, ..., D]
        (or [B, N*D]), result in that layout (used by TracedWideModel)."""
        return ops.layernorm_packed(x, self.weight, self.bias, self.n, self.normalized_shape, self.eps)

    @classmethod
    def from_modules(cls, modules: List[nn.LayerNorm]) -> 'WideLayerNorm':
        t = modules[0]
        shape = t.normalized_shape
        if isinstance(shape, (tuple, list)):
            if len(shape) != 1:
                raise ValueError("WideLayerNorm supports a 1-D normalized_shape only")
            shape = shape[0]
        if t.weight is None or t.bias is None:
            raise ValueError("WideLayerNorm.from_modules needs elementwise_affine=True LayerNorms")
        wide = cls(len(modules), int(shape), t.eps).to(device=t.weight.device, dtype=t.weight.dtype)
        with torch.no_grad():
            wide.weight.copy_(torch.cat([m.weight for m in modules]))
            wide.bias.copy_(torch.cat([m.bias for m in modules]))
        return wide

    def __repr__(self):
        return f"WideLayerNorm({self.n}x{self.normalized_shape})"


__all__ = ['WideLayerNorm']
