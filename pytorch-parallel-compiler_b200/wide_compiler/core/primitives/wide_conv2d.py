"""WideConv2d: N independent Conv2d layers as one implicit-GEMM kernel.

Parameter layout as the reference (wide_conv2d.py:149-158): an inner grouped
``nn.Conv2d(N*Cin, N*Cout, groups=N)`` named ``grouped_conv`` holds the
weights [N*Cout, Cin, kh, kw] and bias [N*Cout]; it is storage only. Forward
[N, B, Cin, H, W] -> [N, B, Cout, H', W'] contiguous (reference :169-194),
computed directly on the N-first layout (no channel-packing copies).
"""
from __future__ import annotations

import warnings
from enum import Enum
from typing import List, Tuple, Union

import torch
from torch import Tensor, nn

from ... import ops
from ._conv_common import check_padding, ntuple


class ConvStrategy(Enum):
    AUTO = 'auto'
    GROUPED = 'grouped'
    CHANNELS_LAST = 'channels_last'
    SEQUENTIAL = 'sequential'


STRATEGY_THRESHOLDS = {'n_high': 16, 'n_crossover': 8, 'n_low': 3, 'b_low': 16}

_WARNED_ABOUT_TUNING = False


def select_strategy(n: int, b: int, c_in: int, c_out: int, h: int = 56, w: int = 56) -> ConvStrategy:
    """Reference heuristic (wide_conv2d.py:67-96), kept for API parity.

    Like the reference it warns once that the thresholds are hardware-tuned.
    """
    global _WARNED_ABOUT_TUNING
    if not _WARNED_ABOUT_TUNING:
        warnings.warn("WideConv2d auto-selection thresholds may need tuning for your GPU. "
                      "Run the test suite to verify optimal strategy for your hardware.", UserWarning)
        _WARNED_ABOUT_TUNING = True
    t = STRATEGY_THRESHOLDS
    if n <= t['n_low']:
        return ConvStrategy.SEQUENTIAL
    if (n >= t['n_crossover'] and b <= t['b_low']) or n >= t['n_high']:
        return ConvStrategy.GROUPED
    return ConvStrategy.SEQUENTIAL


class WideConv2d(nn.Module):
    """N parallel Conv2d layers; N-first input and output."""

    def __init__(self, n: int, in_channels: int, out_channels: int,
                 kernel_size: Union[int, Tuple[int, int]], stride: Union[int, Tuple[int, int]] = 1,
                 padding: Union[int, Tuple[int, int]] = 0, dilation: Union[int, Tuple[int, int]] = 1,
                 bias: bool = True, strategy: Union[str, ConvStrategy] = 'auto'):
        super().__init__()
        check_padding(padding)
        self.n = n
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = ntuple(kernel_size, 2)
        self.stride = ntuple(stride, 2)
        self.padding = ntuple(padding, 2)
        self.dilation = ntuple(dilation, 2)
        self.has_bias = bias
        if isinstance(strategy, str):
            strategy = ConvStrategy(strategy)
        if strategy == ConvStrategy.AUTO:
            strategy = select_strategy(n, 8, in_channels, out_channels, 56, 56)
        self._strategy = strategy
        self._use_grouped = strategy == ConvStrategy.GROUPED
        self._use_channels_last = strategy == ConvStrategy.CHANNELS_LAST
        self.grouped_conv = nn.Conv2d(n * in_channels, n * out_channels, self.kernel_size, stride=self.stride,
                                      padding=self.padding, dilation=self.dilation, groups=n, bias=bias)

    @property
    def strategy(self) -> ConvStrategy:
        return self._strategy

    def forward(self, x: Tensor) -> Tensor:
        return ops.conv_nd(x, self.grouped_conv.weight, self.grouped_conv.bias, self.n,
                           self.stride, self.padding, self.dilation)

    @classmethod
    def from_modules(cls, modules: List[nn.Conv2d], strategy: Union[str, ConvStrategy] = 'auto') -> 'WideConv2d':
        t = modules[0]
        if t.groups != 1:
            raise ValueError("WideConv2d.from_modules supports groups=1 convolutions")
        check_padding(t.padding)
        wide = cls(len(modules), t.in_channels, t.out_channels, ntuple(t.kernel_size, 2), ntuple(t.stride, 2),
                   ntuple(t.padding, 2), ntuple(t.dilation, 2), bias=t.bias is not None, strategy=strategy)
        wide = wide.to(device=t.weight.device, dtype=t.weight.dtype)
        with torch.no_grad():
            wide.grouped_conv.weight.copy_(torch.cat([m.weight for m in modules]))
            if wide.grouped_conv.bias is not None:
                wide.grouped_conv.bias.copy_(torch.cat([m.bias for m in modules]))
        return wide

    def __repr__(self):
        return (f"WideConv2d({self.n}x[{self.in_channels}->{self.out_channels}], "
                f"k={self.kernel_size}, strategy={self._strategy.value})")


__all__ = ['WideConv2d', 'ConvStrategy', 'select_strategy', 'STRATEGY_THRESHOLDS']
