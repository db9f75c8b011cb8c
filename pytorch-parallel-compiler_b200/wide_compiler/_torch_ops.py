"""The wide ops as torch.library custom operators (namespace ``widek``).

Each operator's implementation is the kernel path of ``ops`` (libwidek
through its C-ABI); its fake implementation states the outputs' shapes,
dtypes and devices without running anything; its autograd formula re-runs
the op's torch formulation (``_autograd``) on the saved inputs. With them
dynamo can trace a wide module into one graph of opaque kernel calls, as
the reference's quick start does with
``torch.compile(WideGRU.from_modules(grus), mode='reduce-overhead')``
(reference README.md:65; wide_compiler/api.py:137-147 compiles a
TracedWideModel the same way).

The primitives reach these operators only while dynamo traces
(``torch.compiler.is_compiling()``, checked at the top of each ``ops``
function); eager calls go straight to the kernels. ``widek::batchnorm``
updates the running statistics in place (declared as mutated) and has no
autograd formula under torch.compile: training-mode BatchNorm with
gradients runs eagerly.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
from torch import Tensor

from . import _autograd as _AG
from . import ops


def _register_autograd(op, torch_fn) -> None:
    """Backward of ``op``: gradients of ``torch_fn`` (same argument order)
    with respect to the tensor inputs that need them."""

    def setup_context(ctx, inputs, output):
        ctx.kinds = [isinstance(i, Tensor) for i in inputs]
        ctx.consts = [None if isinstance(i, Tensor) else i for i in inputs]
        ctx.save_for_backward(*[i for i in inputs if isinstance(i, Tensor)])

    def backward(ctx, *grads):
        saved = iter(ctx.saved_tensors)
        args = [next(saved) if k else c for k, c in zip(ctx.kinds, ctx.consts)]
        with torch.enable_grad():
            det = [a.detach().requires_grad_(bool(need) and a.is_floating_point()) if isinstance(a, Tensor) else a
                   for a, need in zip(args, ctx.needs_input_grad)]
            out = torch_fn(*det)
            outs = out if isinstance(out, tuple) else (out,)
            pairs = [(o, g) for o, g in zip(outs, grads) if g is not None and o.requires_grad]
            wanted = [a for a in det if isinstance(a, Tensor) and a.requires_grad]
            got = (torch.autograd.grad([o for o, _ in pairs], wanted, [g for _, g in pairs], allow_unused=True)
                   if pairs and wanted else [None] * len(wanted))
        it = iter(got)
        return tuple(next(it) if isinstance(a, Tensor) and a.requires_grad else None for a in det)

    op.register_autograd(backward, setup_context=setup_context)


# ---------------------------------------------------------------------------
# Operators
# ---------------------------------------------------------------------------

@torch.library.custom_op("widek::linear", mutates_args=())
def linear(x: Tensor, weight: Tensor, bias: Optional[Tensor], act: int) -> Tensor:
    """WideLinear (wide_linear.py:165-168): act(x[i] @ weight[i]^T + bias[i])."""
    with torch.no_grad():
        return ops.linear(x, weight, bias, act)


@linear.register_fake
def _(x, weight, bias, act):
    return x.new_empty((*x.shape[:-1], weight.shape[1]))


_register_autograd(linear, _AG.linear_t)


@torch.library.custom_op("widek::layernorm", mutates_args=())
def layernorm(x: Tensor, weight: Tensor, bias: Tensor, n: int, d: int, eps: float) -> Tensor:
    """WideLayerNorm (wide_layernorm.py:62-65)."""
    with torch.no_grad():
        return ops.layernorm(x, weight, bias, n, d, eps)


@layernorm.register_fake
def _(x, weight, bias, n, d, eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


_register_autograd(layernorm, _AG.layernorm_t)


@torch.library.custom_op("widek::batchnorm", mutates_args=("running_mean", "running_var"))
def batchnorm(x: Tensor, n: int, c: int, weight: Optional[Tensor], bias: Optional[Tensor],
              running_mean: Optional[Tensor], running_var: Optional[Tensor], use_batch_stats: bool,
              update_running: bool, momentum: float, eps: float) -> Tensor:
    """WideBatchNorm1d/2d (wide_batchnorm_2d.py:53-72): running statistics
    updated in place when use_batch_stats and update_running."""
    with torch.no_grad():
        return ops.batchnorm(x, n, c, weight, bias, running_mean, running_var, use_batch_stats, update_running,
                             momentum, eps)


@batchnorm.register_fake
def _(x, n, c, weight, bias, running_mean, running_var, use_batch_stats, update_running, momentum, eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("widek::groupnorm", mutates_args=())
def groupnorm(x: Tensor, n: int, groups: int, weight: Optional[Tensor], bias: Optional[Tensor],
              eps: float) -> Tensor:
    """WideGroupNorm / WideInstanceNorm (wide_groupnorm.py:90-117)."""
    with torch.no_grad():
        return ops.groupnorm(x, n, groups, weight, bias, eps)


@groupnorm.register_fake
def _(x, n, groups, weight, bias, eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


_register_autograd(groupnorm, _AG.groupnorm_t)


@torch.library.custom_op("widek::embedding", mutates_args=())
def embedding(idx: Tensor, weight: Tensor) -> Tensor:
    """WideEmbedding (wide_embedding.py:85-99): weight[:, idx]."""
    with torch.no_grad():
        return ops.embedding(idx, weight)


@embedding.register_fake
def _(idx, weight):
    return weight.new_empty((weight.shape[0], *idx.shape, weight.shape[2]))


_register_autograd(embedding, _AG.embedding_t)


@torch.library.custom_op("widek::conv", mutates_args=())
def conv(x: Tensor, weight: Tensor, bias: Optional[Tensor], n: int, stride: List[int], padding: List[int],
         dilation: List[int]) -> Tensor:
    """WideConv1d/2d/3d (wide_conv2d.py:169-194) on the N-first layout."""
    with torch.no_grad():
        return ops.conv_nd(x, weight, bias, n, tuple(stride), tuple(padding), tuple(dilation))


@conv.register_fake
def _(x, weight, bias, n, stride, padding, dilation):
    nd = x.dim() - 3
    ks = weight.shape[2:]
    osp = [(x.shape[3 + i] + 2 * padding[i] - dilation[i] * (ks[i] - 1) - 1) // stride[i] + 1 for i in range(nd)]
    return x.new_empty((n, x.shape[1], weight.shape[0] // n, *osp))


_register_autograd(conv, lambda x, w, b, n, st, pd, dl: _AG.conv_nd_t(x, w, b, n, tuple(st), tuple(pd), tuple(dl)))


@torch.library.custom_op("widek::gru", mutates_args=())
def gru(x: Tensor, h0: Optional[Tensor], w_ih: Tensor, w_hh: Tensor, b_ih: Optional[Tensor],
        b_hh: Optional[Tensor]) -> Tuple[Tensor, Tensor]:
    """WideGRU (wide_gru.py:148-213): (out [N, B, T, H], h_n [N, B, H])."""
    with torch.no_grad():
        return ops.gru(x, h0, w_ih, w_hh, b_ih, b_hh)


@gru.register_fake
def _(x, h0, w_ih, w_hh, b_ih, b_hh):
    n, b, t, _ = x.shape
    h = w_hh.shape[2]
    return x.new_empty((n, b, t, h)), x.new_empty((n, b, h))


_register_autograd(gru, _AG.gru_t)


def _lstm_blockdiag_t(x, h0, c0, weight_ih, weight_hh, b_ih, b_hh, n, hidden):
    """Torch formulation of the block-diagonal LSTM (wide_lstm.py:184-234)."""
    inp = x.shape[3]
    idx = torch.arange(n, device=x.device)
    wih = weight_ih.view(n, 4 * hidden, n, inp)[idx, :, idx, :]
    whh = weight_hh.view(n, 4 * hidden, n, hidden)[idx, :, idx, :]
    return _AG.lstm_t(x, h0, c0, wih, whh, b_ih, b_hh)


@torch.library.custom_op("widek::lstm", mutates_args=())
def lstm(x: Tensor, h0: Optional[Tensor], c0: Optional[Tensor], weight_ih: Tensor, weight_hh: Tensor,
         b_ih: Optional[Tensor], b_hh: Optional[Tensor], n: int, hidden: int) -> Tuple[Tensor, Tensor, Tensor]:
    """WideLSTM (wide_lstm.py:158-234) from its block-diagonal parameters:
    (out [N, B, T, H], h_n, c_n [N, B, H])."""
    with torch.no_grad():
        out, (hn, cn) = ops.lstm_blockdiag(x, h0, c0, weight_ih, weight_hh, b_ih, b_hh, n, hidden)
        return out, hn, cn


@lstm.register_fake
def _(x, h0, c0, weight_ih, weight_hh, b_ih, b_hh, n, hidden):
    b, t = x.shape[1], x.shape[2]
    return x.new_empty((n, b, t, hidden)), x.new_empty((n, b, hidden)), x.new_empty((n, b, hidden))


_register_autograd(lstm, _lstm_blockdiag_t)


@torch.library.custom_op("widek::attention", mutates_args=())
def attention(query: Tensor, key: Tensor, value: Tensor, q_weight: Tensor, q_bias: Optional[Tensor],
              kv_weight: Tensor, kv_bias: Optional[Tensor], out_weight: Tensor, out_bias: Optional[Tensor],
              n_heads: int, attn_mask: Optional[Tensor], is_causal: bool, self_attn: bool) -> Tensor:
    """WideAttention (wide_attention.py:178-238) on N-first tensors."""
    with torch.no_grad():
        return ops.attention_tensors(query, key, value, q_weight, q_bias, kv_weight, kv_bias, out_weight, out_bias,
                                     n_heads, attn_mask, is_causal, self_attn)


@attention.register_fake
def _(query, key, value, q_weight, q_bias, kv_weight, kv_bias, out_weight, out_bias, n_heads, attn_mask, is_causal,
      self_attn):
    return query.new_empty((*query.shape[:3], out_weight.shape[1]))


_register_autograd(attention, lambda q, k, v, qw, qb, kvw, kvb, ow, ob, h, m, c, s:
                   _AG.attention_t(q, k, v, m, c, h, qw, qb, kvw, kvb, ow, ob))


@torch.library.custom_op("widek::swap01", mutates_args=())
def swap01(x: Tensor) -> Tensor:
    """The TracedWideModel boundary layout change (traced_wide.py:463-469, :531-532)."""
    with torch.no_grad():
        return ops.swap01(x)


@swap01.register_fake
def _(x):
    return x.new_empty((x.shape[1], x.shape[0], *x.shape[2:]))


_register_autograd(swap01, _AG.swap01_t)


@torch.library.custom_op("widek::unary", mutates_args=())
def unary(x: Tensor, op: str) -> Tensor:
    """Elementwise glue (traced_wide.py:174-186): relu / gelu / sigmoid / tanh / silu."""
    with torch.no_grad():
        return ops.unary(x, op)


@unary.register_fake
def _(x, op):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


_register_autograd(unary, _AG.unary_t)


@torch.library.custom_op("widek::binary", mutates_args=())
def binary(a: Tensor, b: Tensor, op: str) -> Tensor:
    """Same-shape glue (traced_wide.py:189-211): add / mul / sub / div."""
    with torch.no_grad():
        return ops.binary(a, b, op)


@binary.register_fake
def _(a, b, op):
    return torch.empty_like(a, memory_format=torch.contiguous_format)


_register_autograd(binary, _AG.binary_t)


OPERATORS = ('linear', 'layernorm', 'batchnorm', 'groupnorm', 'embedding', 'conv', 'gru', 'lstm', 'attention',
             'swap01', 'unary', 'binary')

__all__ = ['OPERATORS']
