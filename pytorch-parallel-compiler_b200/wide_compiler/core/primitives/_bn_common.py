"""Shared forward for the wide BatchNorms: per-(model, channel) statistics on
the N-first layout, torch.nn.BatchNorm semantics for train/eval and for the
running-statistics update (momentum, or cumulative average when momentum is
None; unbiased variance in the running estimate; num_batches_tracked)."""
from __future__ import annotations

from torch import Tensor, nn

from ... import ops


def wide_batchnorm_forward(x: Tensor, bn: nn.modules.batchnorm._BatchNorm, n: int, c: int) -> Tensor:
    use_batch_stats = bn.training or (bn.running_mean is None and bn.running_var is None)
    factor = 0.0
    if bn.training and bn.track_running_stats and bn.num_batches_tracked is not None:
        bn.num_batches_tracked.add_(1)
        factor = (1.0 / float(bn.num_batches_tracked)) if bn.momentum is None else bn.momentum
    update = bn.training and bn.running_mean is not None
    return ops.batchnorm(x, n, c, bn.weight, bn.bias, bn.running_mean, bn.running_var,
                         use_batch_stats=use_batch_stats, update_running=update, momentum=factor, eps=bn.eps)
