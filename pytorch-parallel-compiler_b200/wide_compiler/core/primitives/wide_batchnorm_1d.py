"""WideBatchNorm1d: N BatchNorm1d(C) on [N, B, C] or [N, B, C, L].

Parameter/buffer layout as the reference (wide_batchnorm_1d.py:21-51): an
inner ``op = nn.BatchNorm1d(N*C)``. Forward semantics as reference :53-73.
"""
from __future__ import annotations

from typing import List

from torch import Tensor, nn

from ._bn_common import wide_batchnorm_forward
from .wide_batchnorm_2d import _bn_from_modules


class WideBatchNorm1d(nn.Module):
    def __init__(self, n: int, num_features: int, eps: float = 1e-5, momentum: float = 0.1, affine: bool = True,
                 track_running_stats: bool = True):
        super().__init__()
        self.n = n
        self.num_features = num_features
        self.op = nn.BatchNorm1d(n * num_features, eps=eps, momentum=momentum, affine=affine,
                                 track_running_stats=track_running_stats)

    def forward(self, x: Tensor) -> Tensor:
        if x.dim() not in (3, 4):
            raise ValueError(f"WideBatchNorm1d expects [N, B, C] or [N, B, C, L], got {tuple(x.shape)}")
        return wide_batchnorm_forward(x, self.op, self.n, self.num_features)

    def forward_packed(self, x: Tensor):
        """The same BatchNorm on the packed boundary layout [B, N*C] or
        [B, N*C, L], run as one model of N*C channels (see WideBatchNorm2d)."""
        if x.dim() not in (2, 3):
            return None
        return wide_batchnorm_forward(x.unsqueeze(0), self.op, 1, self.n * self.num_features).squeeze(0)

    @classmethod
    def from_modules(cls, modules: List[nn.BatchNorm1d]) -> 'WideBatchNorm1d':
        return _bn_from_modules(cls, modules)

    def __repr__(self):
        return f"WideBatchNorm1d({self.n}x{self.num_features})"


__all__ = ['WideBatchNorm1d']
