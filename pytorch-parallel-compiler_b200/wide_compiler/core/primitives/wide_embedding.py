"""WideEmbedding: N embedding tables looked up with one shared index tensor.

Parameter layout as the reference (wide_embedding.py:33-80): ``weight``
[N, V, D], N(0, 1) init. Forward: indices [B, T] (any shape) -> [N, B, T, D]
(reference :85-131), one vectorised gather kernel.
"""
from __future__ import annotations

from enum import Enum
from typing import List, Union

import torch
from torch import Tensor, nn

from ... import ops


class EmbeddingStrategy(Enum):
    INDEXED = 'indexed'
    GATHER = 'gather'
    SEQUENTIAL = 'sequential'
    AUTO = 'auto'


class WideEmbedding(nn.Module):
    def __init__(self, n: int, num_embeddings: int, embedding_dim: int,
                 strategy: Union[str, EmbeddingStrategy] = 'auto'):
        super().__init__()
        self.n = n
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        if isinstance(strategy, str):
            strategy = EmbeddingStrategy(strategy)
        if strategy == EmbeddingStrategy.AUTO:
            strategy = EmbeddingStrategy.INDEXED
        self._strategy = strategy
        self._use_indexed = strategy == EmbeddingStrategy.INDEXED
        self._use_gather = strategy == EmbeddingStrategy.GATHER
        self.weight = nn.Parameter(torch.empty(n, num_embeddings, embedding_dim))
        self._reset_parameters()

    @property
    def strategy(self) -> EmbeddingStrategy:
        return self._strategy

    def _reset_parameters(self):
        nn.init.normal_(self.weight)

    def forward(self, x: Tensor) -> Tensor:
        return ops.embedding(x, self.weight)

    @classmethod
    def from_modules(cls, modules: List[nn.Embedding],
                     strategy: Union[str, EmbeddingStrategy] = 'auto') -> 'WideEmbedding':
        t = modules[0]
        wide = cls(len(modules), t.num_embeddings, t.embedding_dim, strategy=strategy)
        wide = wide.to(device=t.weight.device, dtype=t.weight.dtype)
        with torch.no_grad():
            wide.weight.copy_(torch.stack([m.weight for m in modules]))
        return wide

    def __repr__(self):
        return (f"WideEmbedding({self.n}x[{self.num_embeddings}, {self.embedding_dim}], "
                f"strategy={self._strategy.value})")


__all__ = ['WideEmbedding', 'EmbeddingStrategy']
