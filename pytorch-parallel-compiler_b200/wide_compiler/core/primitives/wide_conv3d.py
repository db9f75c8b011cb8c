"""WideConv3d: N independent Conv3d layers, N-first [N, B, Cin, D, H, W].

Parameter layout as the reference (wide_conv3d.py:28-100): GROUPED keeps an
inner grouped ``conv = nn.Conv3d``; SEQUENTIAL keeps ``convs`` (N Conv3d).
"""
from __future__ import annotations

from enum import Enum
from typing import List, Tuple, Union

import torch
from torch import Tensor, nn

from ... import ops
from ._conv_common import check_padding, ntuple


class Conv3dStrategy(Enum):
    GROUPED = 'grouped'
    SEQUENTIAL = 'sequential'
    AUTO = 'auto'


class WideConv3d(nn.Module):
    """N parallel Conv3d layers."""

    def __init__(self, n: int, in_channels: int, out_channels: int,
                 kernel_size: Union[int, Tuple[int, int, int]], stride=1, padding=0, dilation=1,
                 bias: bool = True, strategy: Union[str, Conv3dStrategy] = 'auto'):
        super().__init__()
        check_padding(padding)
        self.n = n
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = kernel_size
        self.stride = stride
        self.padding = padding
        self.dilation = dilation
        self.has_bias = bias
        if isinstance(strategy, str):
            strategy = Conv3dStrategy(strategy)
        if strategy == Conv3dStrategy.AUTO:
            strategy = Conv3dStrategy.GROUPED
        self._strategy = strategy
        self._use_grouped = strategy == Conv3dStrategy.GROUPED
        if self._use_grouped:
            self.conv = nn.Conv3d(n * in_channels, n * out_channels, kernel_size, stride=stride, padding=padding,
                                  dilation=dilation, groups=n, bias=bias)
        else:
            self.convs = nn.ModuleList([
                nn.Conv3d(in_channels, out_channels, kernel_size, stride=stride, padding=padding,
                          dilation=dilation, bias=bias) for _ in range(n)])

    @property
    def strategy(self) -> Conv3dStrategy:
        return self._strategy

    def _params(self):
        if self._use_grouped:
            return self.conv.weight, self.conv.bias
        w = torch.cat([c.weight for c in self.convs])
        b = torch.cat([c.bias for c in self.convs]) if self.has_bias else None
        return w, b

    def forward(self, x: Tensor) -> Tensor:
        w, b = self._params()
        return ops.conv_nd(x, w, b, self.n, ntuple(self.stride, 3), ntuple(self.padding, 3),
                           ntuple(self.dilation, 3))

    @classmethod
    def from_modules(cls, modules: List[nn.Conv3d], strategy: Union[str, Conv3dStrategy] = 'auto') -> 'WideConv3d':
        t = modules[0]
        if t.groups != 1:
            raise ValueError("WideConv3d.from_modules supports groups=1 convolutions")
        wide = cls(len(modules), t.in_channels, t.out_channels, t.kernel_size, t.stride, t.padding, t.dilation,
                   bias=t.bias is not None, strategy=strategy)
        wide = wide.to(device=t.weight.device, dtype=t.weight.dtype)
        with torch.no_grad():
            if wide._use_grouped:
                wide.conv.weight.copy_(torch.cat([m.weight for m in modules]))
                if wide.has_bias:
                    wide.conv.bias.copy_(torch.cat([m.bias for m in modules]))
            else:
                for i, m in enumerate(modules):
                    wide.convs[i].load_state_dict(m.state_dict())
        return wide

    def __repr__(self):
        return (f"WideConv3d({self.n}x[{self.in_channels}->{self.out_channels}], "
                f"strategy={self._strategy.value})")


__all__ = ['WideConv3d', 'Conv3dStrategy']
