"""WideLinear: N independent nn.Linear layers run as one grouped GEMM.

Parameter layout (state_dict compatible with the reference,
wide_compiler/core/primitives/wide_linear.py:114-118): ``weight`` [N, out, in],
``bias`` [N, out]. Forward: [N, B, ..., in] -> [N, B, ..., out]
(reference forward :138-173). The contraction and the bias add run in one
libwidek kernel (tcgen05 tensor cores for bf16/f16, fp32 FFMA for fp32).
The strategy enum and its heuristic (:36-69) are kept for API compatibility;
every strategy executes on the same kernel.
"""
from __future__ import annotations

import math
from enum import Enum
from typing import List, Union

import torch
from torch import Tensor, nn

from ... import ops


class LinearStrategy(Enum):
    EINSUM = 'einsum'
    SEQUENTIAL = 'sequential'
    AUTO = 'auto'


LINEAR_THRESHOLDS = {
    'n_min_einsum': 8,
    'b_max_for_low_n': 64,
    'expansion_max': 8.0,
    'vocab_size': 10000,
}


def select_linear_strategy(n: int, b: int, in_features: int, out_features: int) -> LinearStrategy:
    """Reference heuristic (wide_linear.py:50-69), kept for API parity."""
    t = LINEAR_THRESHOLDS
    if n < t['n_min_einsum'] and b > t['b_max_for_low_n']:
        return LinearStrategy.SEQUENTIAL
    if out_features >= t['vocab_size']:
        return LinearStrategy.SEQUENTIAL
    return LinearStrategy.EINSUM


class WideLinear(nn.Module):
    """N parallel Linear layers; input and output are N-first."""

    def __init__(self, n: int, in_features: int, out_features: int, bias: bool = True,
                 strategy: Union[str, LinearStrategy] = 'auto'):
        super().__init__()
        self.n = n
        self.in_features = in_features
        self.out_features = out_features
        self.has_bias = bias
        if isinstance(strategy, str):
            strategy = LinearStrategy(strategy)
        if strategy == LinearStrategy.AUTO:
            strategy = select_linear_strategy(n, 32, in_features, out_features)
        self._strategy = strategy
        self._use_einsum = strategy == LinearStrategy.EINSUM
        self.weight = nn.Parameter(torch.empty(n, out_features, in_features))
        if bias:
            self.bias = nn.Parameter(torch.empty(n, out_features))
        else:
            self.register_parameter('bias', None)
        self._reset_parameters()

    @property
    def strategy(self) -> LinearStrategy:
        return self._strategy

    def _reset_parameters(self):
        # Per model, as nn.Linear does: kaiming-uniform(a=sqrt(5)) weights,
        # U(-1/sqrt(in), 1/sqrt(in)) bias.
        bound = 1.0 / math.sqrt(self.in_features) if self.in_features > 0 else 0.0
        for i in range(self.n):
            nn.init.kaiming_uniform_(self.weight[i], a=math.sqrt(5))
            if self.bias is not None:
                nn.init.uniform_(self.bias[i], -bound, bound)

    def forward(self, x: Tensor) -> Tensor:
        return ops.linear(x, self.weight, self.bias)

    def forward_packed(self, x: Tensor):
        """The same Linear on the packed boundary layout [B, N*T, K] (or
        [B, N*K]): the kernel reads and writes the packed rows in place,
        result [B, N*T, O] (or [B, N*O]); used by TracedWideModel."""
        if x.dim() == 2:
            if x.shape[1] != self.n * self.in_features:
                return None
            y = ops.linear_layout(x.view(x.shape[0], self.n, self.in_features), self.weight, self.bias,
                                  ops.ACT_NONE, True, True)
            return y.view(x.shape[0], self.n * self.out_features)
        if x.dim() != 3 or x.shape[1] % self.n != 0:
            return None
        return ops.linear_layout(x, self.weight, self.bias, ops.ACT_NONE, True, True)

    @classmethod
    def from_modules(cls, modules: List[nn.Linear], strategy: Union[str, LinearStrategy] = 'auto') -> 'WideLinear':
        t = modules[0]
        wide = cls(len(modules), t.in_features, t.out_features, bias=t.bias is not None, strategy=strategy)
        wide = wide.to(device=t.weight.device, dtype=t.weight.dtype)
        with torch.no_grad():
            wide.weight.copy_(torch.stack([m.weight for m in modules]))
            if wide.bias is not None:
                wide.bias.copy_(torch.stack([m.bias for m in modules]))
        return wide

    def __repr__(self):
        return (f"WideLinear({self.n}x[{self.in_features}->{self.out_features}], "
                f"strategy={self._strategy.value})")


__all__ = ['WideLinear', 'LinearStrategy', 'select_linear_strategy', 'LINEAR_THRESHOLDS']
