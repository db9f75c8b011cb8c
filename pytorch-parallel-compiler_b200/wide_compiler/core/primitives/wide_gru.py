"""WideGRU: N single-layer GRUs (batch-first), persistent recurrent kernel.

Parameter layout as the reference (wide_gru.py:101-106): ``weight_ih``
[N, 3H, I], ``weight_hh`` [N, 3H, H], ``bias_ih``/``bias_hh`` [N, 3H]; gate
order r, z, n; U(+-1/sqrt(H)) init (:117-125). Forward [N, B, T, I] with an
optional h_0 [N, B, H] -> (output [N, B, T, H], h_n [N, B, H]) (:127-213).
The input projection for all steps is one grouped GEMM; the 32..T recurrent
steps run inside one kernel launch that keeps W_hh resident on chip.
"""
from __future__ import annotations

import math
from enum import Enum
from typing import List, Optional, Tuple, Union

import torch
from torch import Tensor, nn

from ... import ops


class GRUStrategy(Enum):
    FUSED = 'fused'
    SEQUENTIAL = 'sequential'
    AUTO = 'auto'


class WideGRU(nn.Module):
    def __init__(self, n: int, input_size: int, hidden_size: int, num_layers: int = 1, bias: bool = True,
                 batch_first: bool = True, dropout: float = 0.0, bidirectional: bool = False,
                 strategy: Union[str, GRUStrategy] = 'auto'):
        super().__init__()
        if num_layers != 1:
            raise NotImplementedError("WideGRU only supports num_layers=1 for fused strategy")
        if bidirectional:
            raise NotImplementedError("WideGRU only supports unidirectional for fused strategy")
        self.n = n
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.num_layers = num_layers
        self.has_bias = bias
        self.batch_first = batch_first
        self.dropout = dropout
        self.bidirectional = bidirectional
        if isinstance(strategy, str):
            strategy = GRUStrategy(strategy)
        if strategy == GRUStrategy.AUTO:
            strategy = GRUStrategy.FUSED
        self._strategy = strategy
        self._use_fused = strategy == GRUStrategy.FUSED
        h = hidden_size
        self.weight_ih = nn.Parameter(torch.empty(n, 3 * h, input_size))
        self.weight_hh = nn.Parameter(torch.empty(n, 3 * h, h))
        if bias:
            self.bias_ih = nn.Parameter(torch.empty(n, 3 * h))
            self.bias_hh = nn.Parameter(torch.empty(n, 3 * h))
        else:
            self.register_parameter('bias_ih', None)
            self.register_parameter('bias_hh', None)
        self._reset_parameters()

    @property
    def strategy(self) -> GRUStrategy:
        return self._strategy

    def _reset_parameters(self):
        s = 1.0 / math.sqrt(self.hidden_size)
        for p in self.parameters():
            nn.init.uniform_(p, -s, s)

    def forward(self, x: Tensor, h_0: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
        return ops.gru(x, h_0, self.weight_ih, self.weight_hh, self.bias_ih, self.bias_hh)

    def forward_packed(self, x: Tensor, h_0=None):
        """The same GRU on the packed boundary layout [B, N*T, I]: the kernels
        read the packed input and write the packed output [B, N*T, H] in
        place; h_n stays [N, B, H] (used by TracedWideModel)."""
        if h_0 is not None or x.dim() != 3:
            return None
        return ops.gru_packed(x, self.weight_ih, self.weight_hh, self.bias_ih, self.bias_hh)

    @classmethod
    def from_modules(cls, modules: List[nn.GRU], strategy: Union[str, GRUStrategy] = 'auto') -> 'WideGRU':
        t = modules[0]
        if t.num_layers != 1:
            raise ValueError("WideGRU.from_modules only supports single-layer GRUs")
        if t.bidirectional:
            raise ValueError("WideGRU.from_modules only supports unidirectional GRUs")
        wide = cls(len(modules), t.input_size, t.hidden_size, num_layers=1, bias=t.bias,
                   batch_first=t.batch_first, dropout=t.dropout, bidirectional=False, strategy=strategy)
        p0 = next(t.parameters())
        wide = wide.to(device=p0.device, dtype=p0.dtype)
        with torch.no_grad():
            wide.weight_ih.copy_(torch.stack([m.weight_ih_l0 for m in modules]))
            wide.weight_hh.copy_(torch.stack([m.weight_hh_l0 for m in modules]))
            if t.bias:
                wide.bias_ih.copy_(torch.stack([m.bias_ih_l0 for m in modules]))
                wide.bias_hh.copy_(torch.stack([m.bias_hh_l0 for m in modules]))
        return wide

    def __repr__(self):
        return (f"WideGRU({self.n}x[{self.input_size}->{self.hidden_size}], "
                f"strategy={self._strategy.value})")


__all__ = ['WideGRU', 'GRUStrategy']
