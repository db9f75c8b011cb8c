"""WideLSTM: N single-layer LSTMs (batch-first), persistent recurrent kernel.

Parameter layout as the reference (wide_lstm.py:101-106): block-diagonal
``weight_ih`` [N*4H, N*I], ``weight_hh`` [N*4H, N*H], ``bias_ih``/``bias_hh``
[N*4H]; gate order i, f, g, o. The dense [N, 4H, I] / [N, 4H, H] diagonal
blocks are extracted once and cached until a parameter changes (the reference
re-extracts them on every forward, :184-199). Forward [N, B, T, I] with
optional (h_0, c_0) each [N, B, H] -> (output [N, B, T, H], (h_n, c_n)).
"""
from __future__ import annotations

from enum import Enum
from typing import List, Optional, Tuple, Union

import torch
from torch import Tensor, nn

from ... import _derived, ops


class LSTMStrategy(Enum):
    FUSED = 'fused'
    SEQUENTIAL = 'sequential'
    AUTO = 'auto'


class WideLSTM(nn.Module):
    def __init__(self, n: int, input_size: int, hidden_size: int, num_layers: int = 1, bias: bool = True,
                 batch_first: bool = True, dropout: float = 0.0, bidirectional: bool = False,
                 strategy: Union[str, LSTMStrategy] = 'auto'):
        super().__init__()
        if num_layers != 1:
            raise NotImplementedError("WideLSTM currently only supports num_layers=1")
        if bidirectional:
            raise NotImplementedError("WideLSTM currently only supports bidirectional=False")
        if not batch_first:
            raise NotImplementedError("WideLSTM currently only supports batch_first=True")
        self.n = n
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.num_layers = num_layers
        self.bias = bias
        self.batch_first = batch_first
        self.dropout = dropout
        self.bidirectional = bidirectional
        if isinstance(strategy, str):
            strategy = LSTMStrategy(strategy)
        if strategy == LSTMStrategy.AUTO:
            strategy = LSTMStrategy.FUSED
        self._strategy = strategy
        i, h = input_size, hidden_size
        self.weight_ih = nn.Parameter(torch.empty(n * 4 * h, n * i))
        self.weight_hh = nn.Parameter(torch.empty(n * 4 * h, n * h))
        if bias:
            self.bias_ih = nn.Parameter(torch.empty(n * 4 * h))
            self.bias_hh = nn.Parameter(torch.empty(n * 4 * h))
        else:
            self.register_parameter('bias_ih', None)
            self.register_parameter('bias_hh', None)
        self._init_weights()

    @property
    def strategy(self) -> LSTMStrategy:
        return self._strategy

    def _init_weights(self):
        i, h, n = self.input_size, self.hidden_size, self.n
        s = 1.0 / (h ** 0.5)
        with torch.no_grad():
            self.weight_ih.zero_()
            self.weight_hh.zero_()
            for k in range(n):
                self.weight_ih[k * 4 * h:(k + 1) * 4 * h, k * i:(k + 1) * i].uniform_(-s, s)
                self.weight_hh[k * 4 * h:(k + 1) * 4 * h, k * h:(k + 1) * h].uniform_(-s, s)
            if self.bias:
                self.bias_ih.zero_()
                self.bias_hh.zero_()

    def _blocks(self) -> Tuple[Tensor, Tensor]:
        """Diagonal blocks [N, 4H, I] and [N, 4H, H], kept between forwards
        while the parameters are unchanged (``wide_compiler._derived``:
        rebuilt after in-place updates and inside every CUDA-graph capture);
        built afresh, differentiably, when autograd needs them."""
        if torch.is_grad_enabled() and (self.weight_ih.requires_grad or self.weight_hh.requires_grad):
            n, h, i = self.n, self.hidden_size, self.input_size
            idx = torch.arange(n, device=self.weight_ih.device)
            return (self.weight_ih.view(n, 4 * h, n, i)[idx, :, idx, :],
                    self.weight_hh.view(n, 4 * h, n, h)[idx, :, idx, :])

        def build():
            n, h, i = self.n, self.hidden_size, self.input_size
            with torch.no_grad():
                wih = self.weight_ih.view(n, 4 * h, n, i)
                whh = self.weight_hh.view(n, 4 * h, n, h)
                idx = torch.arange(n, device=self.weight_ih.device)
                return wih[idx, :, idx, :].contiguous(), whh[idx, :, idx, :].contiguous()   # [N, 4H, I], [N, 4H, H]
        return _derived.cached(self, 'blocks', (self.weight_ih, self.weight_hh), build)

    def forward(self, x: Tensor, hx: Optional[Tuple[Tensor, Tensor]] = None
                ) -> Tuple[Tensor, Tuple[Tensor, Tensor]]:
        n, h = self.n, self.hidden_size
        bih = self.bias_ih.view(n, 4 * h) if self.bias else None
        bhh = self.bias_hh.view(n, 4 * h) if self.bias else None
        h0, c0 = (hx[0], hx[1]) if hx is not None else (None, None)
        # Without autograd the kernels read the block-diagonal parameters in
        # place (by stride); the differentiable path uses the diagonal blocks.
        y = ops.lstm_blockdiag(x, h0, c0, self.weight_ih, self.weight_hh, bih, bhh, n, h)
        if y is not None:
            return y
        wih, whh = self._blocks()
        return ops.lstm(x, h0, c0, wih, whh, bih, bhh)

    def forward_packed(self, x: Tensor, hx=None):
        """The same LSTM on the packed boundary layout [B, N*T, I] (packed
        output [B, N*T, H]; h_n, c_n stay [N, B, H]), used by TracedWideModel."""
        if hx is not None or x.dim() != 3:
            return None
        n, h = self.n, self.hidden_size
        bih = self.bias_ih.view(n, 4 * h) if self.bias else None
        bhh = self.bias_hh.view(n, 4 * h) if self.bias else None
        return ops.lstm_blockdiag_packed(x, self.weight_ih, self.weight_hh, bih, bhh, n, h)

    @classmethod
    def from_modules(cls, modules: List[nn.LSTM], strategy: Union[str, LSTMStrategy] = 'auto') -> 'WideLSTM':
        t = modules[0]
        for m in modules:
            if m.input_size != t.input_size or m.hidden_size != t.hidden_size:
                raise ValueError("WideLSTM.from_modules: all LSTMs must share input/hidden sizes")
            if m.num_layers != 1 or m.bidirectional or m.batch_first != t.batch_first:
                raise ValueError("WideLSTM.from_modules: single-layer, unidirectional LSTMs only")
        wide = cls(len(modules), t.input_size, t.hidden_size, num_layers=1, bias=t.bias, batch_first=True,
                   dropout=t.dropout, bidirectional=False, strategy=strategy)
        p0 = next(t.parameters())
        wide = wide.to(device=p0.device, dtype=p0.dtype)
        i, h = t.input_size, t.hidden_size
        with torch.no_grad():
            wide.weight_ih.zero_()
            wide.weight_hh.zero_()
            for k, m in enumerate(modules):
                wide.weight_ih[k * 4 * h:(k + 1) * 4 * h, k * i:(k + 1) * i] = m.weight_ih_l0
                wide.weight_hh[k * 4 * h:(k + 1) * 4 * h, k * h:(k + 1) * h] = m.weight_hh_l0
            if wide.bias:
                wide.bias_ih.copy_(torch.cat([m.bias_ih_l0 for m in modules]))
                wide.bias_hh.copy_(torch.cat([m.bias_hh_l0 for m in modules]))
        return wide

    def __repr__(self):
        return (f"WideLSTM({self.n}x[{self.input_size}->{self.hidden_size}], "
                f"strategy={self._strategy.value})")


__all__ = ['WideLSTM', 'LSTMStrategy']
