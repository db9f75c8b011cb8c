"""WideBatchNorm2d: N BatchNorm2d(C) as one per-(model, channel) kernel.

Parameter/buffer layout as the reference (wide_batchnorm_2d.py:21-51): an
inner ``op = nn.BatchNorm2d(N*C)`` holds weight, bias, running stats and
num_batches_tracked. Forward [N, B, C, H, W] -> same shape (reference
:53-72) without the channel-packing permute copies.
"""
from __future__ import annotations

from typing import List

import torch
from torch import Tensor, nn

from ._bn_common import wide_batchnorm_forward


class WideBatchNorm2d(nn.Module):
    def __init__(self, n: int, num_features: int, eps: float = 1e-5, momentum: float = 0.1, affine: bool = True,
                 track_running_stats: bool = True):
        super().__init__()
        self.n = n
        self.num_features = num_features
        self.op = nn.BatchNorm2d(n * num_features, eps=eps, momentum=momentum, affine=affine,
                                 track_running_stats=track_running_stats)

    def forward(self, x: Tensor) -> Tensor:
        if x.dim() != 5:
            raise ValueError(f"WideBatchNorm2d expects [N, B, C, H, W], got {tuple(x.shape)}")
        return wide_batchnorm_forward(x, self.op, self.n, self.num_features)

    def forward_packed(self, x: Tensor):
        """The same BatchNorm on the packed boundary layout [B, N*C, H, W]:
        there the (model, channel) pairs are the N*C channels of one
        BatchNorm2d (same parameter order), so it runs as one model of N*C
        channels, result in that layout (used by TracedWideModel)."""
        if x.dim() != 4:
            return None
        return wide_batchnorm_forward(x.unsqueeze(0), self.op, 1, self.n * self.num_features).squeeze(0)

    @classmethod
    def from_modules(cls, modules: List[nn.BatchNorm2d]) -> 'WideBatchNorm2d':
        return _bn_from_modules(cls, modules)

    def __repr__(self):
        return f"WideBatchNorm2d({self.n}x{self.num_features})"


def _bn_from_modules(cls, modules):
    t = modules[0]
    wide = cls(len(modules), t.num_features, eps=t.eps, momentum=t.momentum, affine=t.affine,
               track_running_stats=t.track_running_stats)
    wide = wide.to(device=t.weight.device if t.weight is not None else 'cpu',
                   dtype=t.weight.dtype if t.weight is not None else torch.float32)
    with torch.no_grad():
        for name in ('weight', 'bias', 'running_mean', 'running_var'):
            dst = getattr(wide.op, name)
            if dst is not None and getattr(t, name) is not None:
                dst.copy_(torch.cat([getattr(m, name) for m in modules]))
    return wide


__all__ = ['WideBatchNorm2d']
