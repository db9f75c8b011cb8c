"""WideGroupNorm: N GroupNorm(G, C) with statistics per (model, sample, group).

Parameter layout as the reference (wide_groupnorm.py:29-88): FUSED keeps one
``norm = nn.GroupNorm(N*G, N*C)``; SEQUENTIAL keeps ``norms`` (N GroupNorms).
Forward [N, B, C, *S] -> same shape (reference :90-117).
"""
from __future__ import annotations

from enum import Enum
from typing import List, Union

import torch
from torch import Tensor, nn

from ... import ops


class GroupNormStrategy(Enum):
    FUSED = 'fused'
    SEQUENTIAL = 'sequential'
    AUTO = 'auto'


class WideGroupNorm(nn.Module):
    def __init__(self, n: int, num_groups: int, num_channels: int, eps: float = 1e-5, affine: bool = True,
                 strategy: Union[str, GroupNormStrategy] = 'auto'):
        super().__init__()
        if num_channels % num_groups != 0:
            raise ValueError("num_channels must be divisible by num_groups")
        self.n = n
        self.num_groups = num_groups
        self.num_channels = num_channels
        self.eps = eps
        self.affine = affine
        if isinstance(strategy, str):
            strategy = GroupNormStrategy(strategy)
        if strategy == GroupNormStrategy.AUTO:
            strategy = GroupNormStrategy.FUSED
        self._strategy = strategy
        self._use_fused = strategy == GroupNormStrategy.FUSED
        if self._use_fused:
            self.norm = nn.GroupNorm(n * num_groups, n * num_channels, eps=eps, affine=affine)
        else:
            self.norms = nn.ModuleList([nn.GroupNorm(num_groups, num_channels, eps=eps, affine=affine)
                                        for _ in range(n)])

    @property
    def strategy(self) -> GroupNormStrategy:
        return self._strategy

    def _affine(self):
        if not self.affine:
            return None, None
        if self._use_fused:
            return self.norm.weight, self.norm.bias
        return torch.cat([m.weight for m in self.norms]), torch.cat([m.bias for m in self.norms])

    def forward(self, x: Tensor) -> Tensor:
        w, b = self._affine()
        return ops.groupnorm(x, self.n, self.num_groups, w, b, self.eps)

    def forward_packed(self, x: Tensor):
        """The same GroupNorm on the packed boundary layout [B, N*C, *S]: each
        (model, group) is a run of C/G consecutive channels there, so it is
        one GroupNorm of N*G groups over N*C channels, result in that layout
        (used by TracedWideModel)."""
        if x.dim() < 2:
            return None
        w, b = self._affine()
        return ops.groupnorm(x.unsqueeze(0), 1, self.n * self.num_groups, w, b, self.eps).squeeze(0)

    @classmethod
    def from_modules(cls, modules: List[nn.GroupNorm],
                     strategy: Union[str, GroupNormStrategy] = 'auto') -> 'WideGroupNorm':
        t = modules[0]
        wide = cls(len(modules), t.num_groups, t.num_channels, eps=t.eps, affine=t.affine, strategy=strategy)
        if t.affine:
            wide = wide.to(device=t.weight.device, dtype=t.weight.dtype)
        with torch.no_grad():
            if wide.affine and wide._use_fused:
                wide.norm.weight.copy_(torch.cat([m.weight for m in modules]))
                wide.norm.bias.copy_(torch.cat([m.bias for m in modules]))
            elif wide.affine:
                for i, m in enumerate(modules):
                    wide.norms[i].load_state_dict(m.state_dict())
        return wide

    def __repr__(self):
        return (f"WideGroupNorm({self.n}x[groups={self.num_groups}, channels={self.num_channels}], "
                f"strategy={self._strategy.value})")


__all__ = ['WideGroupNorm', 'GroupNormStrategy']
