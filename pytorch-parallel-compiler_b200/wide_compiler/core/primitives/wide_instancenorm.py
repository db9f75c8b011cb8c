"""WideInstanceNorm1d / WideInstanceNorm2d: per-(model, sample, channel)
normalisation over the spatial dims.

Parameter layout as the reference (wide_instancenorm.py:30-160, :163-290):
FUSED keeps ``norm = nn.InstanceNormXd(N*C)``; SEQUENTIAL keeps ``norms``.
Semantics follow torch.nn.InstanceNorm: instance statistics unless the module
tracks running stats and is in eval mode, in which case the running stats are
used; training with tracked stats also updates them.
Runs on the GroupNorm kernel with one group per channel.
"""
from __future__ import annotations

from enum import Enum
from typing import List, Union

import torch
from torch import Tensor, nn

from ... import ops


class InstanceNormStrategy(Enum):
    FUSED = 'fused'
    SEQUENTIAL = 'sequential'
    AUTO = 'auto'


class _WideInstanceNorm(nn.Module):
    _inner = None          # nn.InstanceNorm1d / 2d
    _spatial_dims = 1

    def __init__(self, n: int, num_features: int, eps: float = 1e-5, momentum: float = 0.1, affine: bool = False,
                 track_running_stats: bool = False, strategy: Union[str, InstanceNormStrategy] = 'auto'):
        super().__init__()
        self.n = n
        self.num_features = num_features
        self.eps = eps
        self.momentum = momentum
        self.affine = affine
        self.track_running_stats = track_running_stats
        if isinstance(strategy, str):
            strategy = InstanceNormStrategy(strategy)
        if strategy == InstanceNormStrategy.AUTO:
            strategy = InstanceNormStrategy.FUSED
        self._strategy = strategy
        self._use_fused = strategy == InstanceNormStrategy.FUSED
        inner = type(self)._inner
        if self._use_fused:
            self.norm = inner(n * num_features, eps=eps, momentum=momentum, affine=affine,
                              track_running_stats=track_running_stats)
        else:
            self.norms = nn.ModuleList([inner(num_features, eps=eps, momentum=momentum, affine=affine,
                                              track_running_stats=track_running_stats) for _ in range(n)])

    @property
    def strategy(self) -> InstanceNormStrategy:
        return self._strategy

    def _cat(self, name):
        if self._use_fused:
            return getattr(self.norm, name)
        parts = [getattr(m, name) for m in self.norms]
        return None if parts[0] is None else torch.cat(parts)

    def forward(self, x: Tensor) -> Tensor:
        if x.dim() != 3 + self._spatial_dims:
            raise ValueError(f"{type(self).__name__} expects {3 + self._spatial_dims}-D N-first input, "
                             f"got {tuple(x.shape)}")
        return self._run(x, self.n, self.num_features)

    def forward_packed(self, x: Tensor):
        """The same InstanceNorm on the packed boundary layout [B, N*C, *S]
        (one model of N*C channels there: the parameters and statistics are
        per (model, channel) either way), result in that layout (used by
        TracedWideModel)."""
        if x.dim() != 2 + self._spatial_dims:
            return None
        return self._run(x.unsqueeze(0), 1, self.n * self.num_features).squeeze(0)

    def _run(self, x: Tensor, n: int, c: int) -> Tensor:
        w, b = (self._cat('weight'), self._cat('bias')) if self.affine else (None, None)
        if self.track_running_stats and not self.training:
            return ops.batchnorm(x, n, c, w, b, self._cat('running_mean'), self._cat('running_var'),
                                 use_batch_stats=False, update_running=False, momentum=0.0, eps=self.eps)
        if self.track_running_stats and self.training:
            if not self._use_fused:
                raise NotImplementedError("running-stat update for the sequential InstanceNorm layout")
            return ops.instancenorm_train(x, n, c, w, b, self.norm.running_mean, self.norm.running_var,
                                          self.momentum, self.eps)
        return ops.groupnorm(x, n, c, w, b, self.eps)

    @classmethod
    def from_modules(cls, modules, strategy: Union[str, InstanceNormStrategy] = 'auto'):
        t = modules[0]
        wide = cls(len(modules), t.num_features, eps=t.eps, momentum=t.momentum, affine=t.affine,
                   track_running_stats=t.track_running_stats, strategy=strategy)
        if t.affine:
            wide = wide.to(device=t.weight.device, dtype=t.weight.dtype)
            with torch.no_grad():
                if wide._use_fused:
                    wide.norm.weight.copy_(torch.cat([m.weight for m in modules]))
                    wide.norm.bias.copy_(torch.cat([m.bias for m in modules]))
                else:
                    for i, m in enumerate(modules):
                        wide.norms[i].load_state_dict(m.state_dict())
        return wide

    def __repr__(self):
        return f"{type(self).__name__}({self.n}x[{self.num_features}], strategy={self._strategy.value})"


class WideInstanceNorm1d(_WideInstanceNorm):
    """N parallel InstanceNorm1d on [N, B, C, L]."""
    _inner = nn.InstanceNorm1d
    _spatial_dims = 1


class WideInstanceNorm2d(_WideInstanceNorm):
    """N parallel InstanceNorm2d on [N, B, C, H, W]."""
    _inner = nn.InstanceNorm2d
    _spatial_dims = 2


__all__ = ['WideInstanceNorm1d', 'WideInstanceNorm2d', 'InstanceNormStrategy']
