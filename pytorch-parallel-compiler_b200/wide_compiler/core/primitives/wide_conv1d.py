"""WideConv1d: N independent Conv1d layers, N-first [N, B, Cin, L].

Parameter layout follows the reference's strategy split
(wide_conv1d.py:38-135): GROUPED keeps an inner grouped ``op = nn.Conv1d``
([N*Cout, Cin, K]); SEQUENTIAL keeps ``weight`` [N, Cout, Cin, K] and ``bias``
[N, Cout]. Both are the same memory layout and run the same kernel.
"""
from __future__ import annotations

import math
from enum import Enum, auto
from typing import List, Optional

import torch
from torch import Tensor, nn

from ... import ops
from ._conv_common import check_padding, ntuple


class Conv1dStrategy(Enum):
    GROUPED = auto()
    SEQUENTIAL = auto()


_GROUPED_THRESHOLD = 10


class WideConv1d(nn.Module):
    """N parallel Conv1d layers."""

    def __init__(self, n: int, in_channels: int, out_channels: int, kernel_size: int, stride: int = 1,
                 padding: int = 0, dilation: int = 1, bias: bool = True,
                 strategy: Optional[Conv1dStrategy] = None):
        super().__init__()
        check_padding(padding)
        self.n = n
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = ntuple(kernel_size, 1)[0]
        self.stride = ntuple(stride, 1)[0]
        self.padding = ntuple(padding, 1)[0]
        self.dilation = ntuple(dilation, 1)[0]
        self.has_bias = bias
        if strategy is None:
            strategy = Conv1dStrategy.GROUPED if n >= _GROUPED_THRESHOLD else Conv1dStrategy.SEQUENTIAL
        self.strategy = strategy
        if strategy == Conv1dStrategy.GROUPED:
            self.op = nn.Conv1d(n * in_channels, n * out_channels, self.kernel_size, stride=self.stride,
                                padding=self.padding, dilation=self.dilation, groups=n, bias=bias)
        else:
            self.weight = nn.Parameter(torch.empty(n, out_channels, in_channels, self.kernel_size))
            if bias:
                self.bias = nn.Parameter(torch.empty(n, out_channels))
            else:
                self.register_parameter('bias', None)
            bound = 1.0 / math.sqrt(in_channels * self.kernel_size)
            for i in range(n):
                nn.init.kaiming_uniform_(self.weight[i], a=math.sqrt(5))
                if bias:
                    nn.init.uniform_(self.bias[i], -bound, bound)

    def _params(self):
        if self.strategy == Conv1dStrategy.GROUPED:
            return self.op.weight, self.op.bias
        w = self.weight.reshape(self.n * self.out_channels, self.in_channels, self.kernel_size)
        b = self.bias.reshape(-1) if self.bias is not None else None
        return w, b

    def forward(self, x: Tensor) -> Tensor:
        w, b = self._params()
        return ops.conv_nd(x, w, b, self.n, (self.stride,), (self.padding,), (self.dilation,))

    @classmethod
    def from_modules(cls, modules: List[nn.Conv1d], strategy: Optional[Conv1dStrategy] = None) -> 'WideConv1d':
        t = modules[0]
        if t.groups != 1:
            raise ValueError("WideConv1d.from_modules supports groups=1 convolutions")
        check_padding(t.padding)
        wide = cls(len(modules), t.in_channels, t.out_channels, ntuple(t.kernel_size, 1)[0],
                   ntuple(t.stride, 1)[0], ntuple(t.padding, 1)[0], ntuple(t.dilation, 1)[0],
                   bias=t.bias is not None, strategy=strategy)
        wide = wide.to(device=t.weight.device, dtype=t.weight.dtype)
        with torch.no_grad():
            w = torch.stack([m.weight for m in modules])
            if wide.strategy == Conv1dStrategy.GROUPED:
                wide.op.weight.copy_(w.reshape_as(wide.op.weight))
                if t.bias is not None:
                    wide.op.bias.copy_(torch.cat([m.bias for m in modules]))
            else:
                wide.weight.copy_(w)
                if t.bias is not None:
                    wide.bias.copy_(torch.stack([m.bias for m in modules]))
        return wide

    def __repr__(self):
        return (f"WideConv1d({self.n}x[{self.in_channels}->{self.out_channels}], k={self.kernel_size}, "
                f"strategy={self.strategy.name})")


__all__ = ['WideConv1d', 'Conv1dStrategy']
