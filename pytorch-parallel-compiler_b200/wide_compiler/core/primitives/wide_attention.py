"""WideAttention: N independent multi-head attention modules.

Parameter layout as the reference (wide_attention.py:98-114): ``q_weight``
[N, D, D], ``kv_weight`` [N, 2D, D] (K rows first, then V), ``q_bias`` [N, D],
``kv_bias`` [N, 2D], ``out_weight`` [N, D, D], ``out_bias`` [N, D]; xavier
init per model (:122-136). Forward on N-first [N, B, T, D]; returns a tuple
``(out, None)`` when key is passed (MHA-style call) and a tensor otherwise
(:138-176). Scaled dot-product attention with scale 1/sqrt(head_dim),
optional causal masking or an additive/boolean [Tq, Tkv] mask.

Kernels: the Q/K/V projections are one grouped GEMM over the concatenated
[q; kv] weight for self-attention (separate GEMMs for cross-attention), the
core is a flash-style kernel reading Q/K/V in place (no head-split copies),
and the output projection is a grouped GEMM with the bias in its epilogue.
"""
from __future__ import annotations

from enum import Enum
from typing import List, Optional, Tuple, Union

import torch
from torch import Tensor, nn

from ... import ops


class AttentionStrategy(Enum):
    FUSED = 'fused'
    SEQUENTIAL = 'sequential'
    AUTO = 'auto'


class WideAttention(nn.Module):
    def __init__(self, n: int, d_model: int, n_heads: int, dropout: float = 0.0, bias: bool = True,
                 strategy: Union[str, AttentionStrategy] = 'auto'):
        super().__init__()
        assert d_model % n_heads == 0, f"d_model ({d_model}) must be divisible by n_heads ({n_heads})"
        self.n = n
        self.d_model = d_model
        self.n_heads = n_heads
        self.d_head = d_model // n_heads
        self.dropout = dropout
        self.has_bias = bias
        if isinstance(strategy, str):
            strategy = AttentionStrategy(strategy)
        if strategy == AttentionStrategy.AUTO:
            strategy = AttentionStrategy.FUSED
        self._strategy = strategy
        self._use_fused = strategy == AttentionStrategy.FUSED
        self.q_weight = nn.Parameter(torch.empty(n, d_model, d_model))
        self.kv_weight = nn.Parameter(torch.empty(n, 2 * d_model, d_model))
        if bias:
            self.q_bias = nn.Parameter(torch.empty(n, d_model))
            self.kv_bias = nn.Parameter(torch.empty(n, 2 * d_model))
        else:
            self.register_parameter('q_bias', None)
            self.register_parameter('kv_bias', None)
        self.out_weight = nn.Parameter(torch.empty(n, d_model, d_model))
        if bias:
            self.out_bias = nn.Parameter(torch.empty(n, d_model))
        else:
            self.register_parameter('out_bias', None)
        self._reset_parameters()

    @property
    def strategy(self) -> AttentionStrategy:
        return self._strategy

    def _reset_parameters(self):
        d = self.d_model
        for i in range(self.n):
            nn.init.xavier_uniform_(self.q_weight[i])
            nn.init.xavier_uniform_(self.kv_weight[i].view(2, d, d))
            nn.init.xavier_uniform_(self.out_weight[i])
            if self.q_bias is not None:
                nn.init.zeros_(self.q_bias[i])
                nn.init.zeros_(self.kv_bias[i])
                nn.init.zeros_(self.out_bias[i])

    def _fused_qkv(self) -> Tuple[Tensor, Optional[Tensor]]:
        """[q; kv] weight [N, 3D, D] (and bias [N, 3D]) for self-attention,
        kept between forwards while the four parameters are unchanged."""
        return ops.fused_qkv(self.q_weight, self.kv_weight, self.q_bias, self.kv_bias)

    def forward(self, query: Tensor, key: Optional[Tensor] = None, value: Optional[Tensor] = None,
                attn_mask: Optional[Tensor] = None, is_causal: bool = False,
                need_weights: bool = False) -> Union[Tensor, Tuple[Tensor, None]]:
        mha_mode = key is not None
        if key is None:
            key = query
        if value is None:
            value = key
        if self.training and self.dropout > 0.0:
            # random attention dropout: projections on the kernels, the core
            # on torch's SDPA with dropout_p (ops.attention_dropout)
            out = ops.attention_dropout(self, query, key, value, attn_mask, is_causal, self.dropout)
        else:
            out = ops.attention(self, query, key, value, attn_mask, is_causal)
        return (out, None) if mha_mode else out

    def forward_packed(self, query: Tensor, key=None, value=None, attn_mask=None, is_causal: bool = False,
                       need_weights: bool = False):
        """Self-attention on the packed boundary layout [B, N*T, D]: the fused
        QKV projection reads the packed rows in place and the output
        projection writes them packed (used by TracedWideModel); other forms
        (cross-attention, masks) decline."""
        mha_mode = key is not None
        if (key is not None and key is not query) or (value is not None and value is not query) \
                or attn_mask is not None or (self.training and self.dropout > 0.0):
            return None
        if query.dim() != 3 or query.shape[1] % self.n != 0 or query.shape[2] != self.d_model:
            return None
        out = ops.attention_packed(self, query, is_causal)
        return (out, None) if mha_mode else out

    @classmethod
    def from_modules(cls, modules: List[nn.MultiheadAttention],
                     strategy: Union[str, AttentionStrategy] = 'auto') -> 'WideAttention':
        t = modules[0]
        if t.in_proj_weight is None:
            raise ValueError("WideAttention.from_modules needs MultiheadAttention with a packed in_proj_weight "
                             "(kdim == vdim == embed_dim)")
        wide = cls(len(modules), t.embed_dim, t.num_heads, dropout=t.dropout, bias=t.in_proj_bias is not None,
                   strategy=strategy)
        wide = wide.to(device=t.in_proj_weight.device, dtype=t.in_proj_weight.dtype)
        d = t.embed_dim
        with torch.no_grad():
            w = torch.stack([m.in_proj_weight for m in modules])        # [N, 3D, D]
            wide.q_weight.copy_(w[:, :d])
            wide.kv_weight.copy_(w[:, d:])
            if t.in_proj_bias is not None:
                b = torch.stack([m.in_proj_bias for m in modules])      # [N, 3D]
                wide.q_bias.copy_(b[:, :d])
                wide.kv_bias.copy_(b[:, d:])
            wide.out_weight.copy_(torch.stack([m.out_proj.weight for m in modules]))
            if t.out_proj.bias is not None and wide.out_bias is not None:
                wide.out_bias.copy_(torch.stack([m.out_proj.bias for m in modules]))
        return wide

    def __repr__(self):
        return (f"WideAttention({self.n}x[d={self.d_model}, h={self.n_heads}], "
                f"strategy={self._strategy.value})")


__all__ = ['WideAttention', 'AttentionStrategy']
