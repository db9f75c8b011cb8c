"""Gradients for the kernel-backed wide ops.

The reference's primitives are plain torch code, so autograd differentiates
them (its LSTM tests check gradient flow, reference
wide_compiler/core/primitives/wide_lstm.py:744-762). Here the forward runs
on the sm_100a kernels; when autograd needs the result (grad mode on and a
tensor argument requiring grad) an op runs through ``Recompute``: the
forward is the kernel, and the backward re-runs the op's torch formulation
below (the reference's own arithmetic, in the storage dtype) on the saved
inputs and differentiates it with ``torch.autograd.grad``. Inference (no
grad needed) never enters this module.

The torch formulations restate, per op, the reference's forward:
  linear       wide_linear.py:162-171 (einsum 'noi,nbi->nbo' + bias)
  layernorm    wide_layernorm.py:62-65
  batchnorm    wide_batchnorm_2d.py:53-72, wide_batchnorm_1d.py:53-73
  groupnorm    wide_groupnorm.py:90-117 (also InstanceNorm, groups = C)
  embedding    wide_embedding.py:85-99
  conv         wide_conv2d.py:169-194 (grouped conv, groups = N)
  attention    wide_attention.py:197-238 (projections, SDPA, out projection)
  gru / lstm   wide_gru.py:168-213, wide_lstm.py:184-234
  glue         traced_wide.py:174-211 (activations, add/mul/sub/div),
               :463-469 / :531-532 (layout changes), ensemble_util.py:45
"""
from __future__ import annotations

import math
from typing import Any, Callable, List, Optional, Sequence

import torch
import torch.nn.functional as F
from torch import Tensor


def needs_grad(*objs: Any) -> bool:
    """Grad mode is on and some tensor argument (also inside a list/tuple)
    requires grad."""
    if not torch.is_grad_enabled():
        return False
    for o in objs:
        if isinstance(o, Tensor):
            if o.requires_grad:
                return True
        elif isinstance(o, (list, tuple)):
            if any(isinstance(t, Tensor) and t.requires_grad for t in o):
                return True
    return False


def _flatten(args: Sequence[Any]):
    """Tensors (top level and inside lists/tuples) and a spec to rebuild the
    argument list around them."""
    tensors: List[Tensor] = []
    spec = []
    for a in args:
        if isinstance(a, Tensor):
            spec.append(('t', len(tensors)))
            tensors.append(a)
        elif isinstance(a, (list, tuple)) and any(isinstance(t, Tensor) for t in a):
            items = []
            for t in a:
                if isinstance(t, Tensor):
                    items.append(('t', len(tensors)))
                    tensors.append(t)
                else:
                    items.append(('v', t))
            spec.append(('l', items))
        else:
            spec.append(('v', a))
    return tensors, spec


def _rebuild(spec, tensors: Sequence[Tensor]):
    out = []
    for kind, val in spec:
        if kind == 't':
            out.append(tensors[val])
        elif kind == 'l':
            out.append([tensors[v] if k == 't' else v for k, v in val])
        else:
            out.append(val)
    return out


class Recompute(torch.autograd.Function):
    """forward: ``kernel_fn(*args)``; backward: gradients of
    ``torch_fn(*args)`` with respect to the tensor arguments. Both functions
    return a tensor or a flat tuple of tensors."""

    @staticmethod
    def forward(ctx, kernel_fn, torch_fn, spec, *tensors):
        ctx.torch_fn, ctx.spec = torch_fn, spec
        ctx.save_for_backward(*tensors)
        with torch.no_grad():
            out = kernel_fn(*_rebuild(spec, tensors))
        if isinstance(out, tuple):
            ctx.mark_non_differentiable(*[o for o in out if not o.is_floating_point()])
        return out

    @staticmethod
    def backward(ctx, *grads):
        saved = ctx.saved_tensors
        with torch.enable_grad():
            inputs = [t.detach().requires_grad_(t.requires_grad and t.is_floating_point()) for t in saved]
            out = ctx.torch_fn(*_rebuild(ctx.spec, inputs))
            outs = out if isinstance(out, tuple) else (out,)
            pairs = [(o, g) for o, g in zip(outs, grads) if g is not None and o.requires_grad]
            wanted = [t for t in inputs if t.requires_grad]
            got = torch.autograd.grad([o for o, _ in pairs], wanted, [g for _, g in pairs],
                                      allow_unused=True) if pairs and wanted else [None] * len(wanted)
        res, it = [], iter(got)
        for t in inputs:
            res.append(next(it) if t.requires_grad else None)
        return (None, None, None, *res)


def run(kernel_fn: Callable, torch_fn: Callable, *args):
    """kernel_fn(*args), made differentiable through torch_fn when needed."""
    if not needs_grad(*args):
        return kernel_fn(*args)
    tensors, spec = _flatten(args)
    return Recompute.apply(kernel_fn, torch_fn, spec, *tensors)


# ---------------------------------------------------------------------------
# Torch formulations (differentiable; the reference's arithmetic)
# ---------------------------------------------------------------------------

def act_t(y: Tensor, act: int) -> Tensor:
    if act == 1:
        return torch.relu(y)
    if act == 2:
        return F.gelu(y)
    return y


def linear_t(x: Tensor, weight: Tensor, bias: Optional[Tensor], act: int = 0, force_simt: bool = False) -> Tensor:
    n, o, k = weight.shape
    y = torch.einsum('noi,nbi->nbo', weight, x.reshape(n, -1, k))
    if bias is not None:
        y = y + bias.unsqueeze(1)
    return act_t(y, act).reshape(*x.shape[:-1], o)


def layernorm_t(x: Tensor, weight: Tensor, bias: Tensor, n: int, d: int, eps: float) -> Tensor:
    shape = (n,) + (1,) * (x.dim() - 2) + (d,)
    return F.layer_norm(x, (d,), eps=eps) * weight.view(shape) + bias.view(shape)


def _chan_view(t: Optional[Tensor], n: int, c: int, dims: int) -> Optional[Tensor]:
    return None if t is None else t.view((n, 1, c) + (1,) * (dims - 3))


def batchnorm_t(x: Tensor, n: int, c: int, weight, bias, running_mean, running_var, use_batch_stats: bool,
                update_running: bool, momentum: float, eps: float) -> Tensor:
    dims = [1] + list(range(3, x.dim()))
    if use_batch_stats:
        mean = x.mean(dim=dims, keepdim=True)
        var = x.var(dim=dims, unbiased=False, keepdim=True)
    else:
        mean = _chan_view(running_mean, n, c, x.dim())
        var = _chan_view(running_var, n, c, x.dim())
    y = (x - mean) / torch.sqrt(var + eps)
    if weight is not None:
        y = y * _chan_view(weight, n, c, x.dim())
    if bias is not None:
        y = y + _chan_view(bias, n, c, x.dim())
    return y


def groupnorm_t(x: Tensor, n: int, groups: int, weight, bias, eps: float, row_stats: bool = False):
    b, c = x.shape[1], x.shape[2]
    xg = x.reshape(n, b, groups, -1)
    mean = xg.mean(dim=-1, keepdim=True)
    var = xg.var(dim=-1, unbiased=False, keepdim=True)
    y = ((xg - mean) / torch.sqrt(var + eps)).reshape(x.shape)
    if weight is not None:
        y = y * _chan_view(weight, n, c, x.dim())
    if bias is not None:
        y = y + _chan_view(bias, n, c, x.dim())
    if row_stats:
        return y, mean.squeeze(-1).float(), var.squeeze(-1).float()
    return y


def embedding_t(idx: Tensor, weight: Tensor) -> Tensor:
    return weight[:, idx.long()]


def swap01_t(x: Tensor) -> Tensor:
    return x.transpose(0, 1).contiguous()


def pack_t(inputs: Sequence[Tensor]) -> Tensor:
    return torch.stack(list(inputs), dim=1)


_UNARY_T = {'relu': torch.relu, 'gelu': F.gelu, 'sigmoid': torch.sigmoid, 'tanh': torch.tanh, 'silu': F.silu}
_BINARY_T = {'add': torch.add, 'mul': torch.mul, 'sub': torch.sub, 'div': torch.div}


def unary_t(x: Tensor, op: str) -> Tensor:
    return _UNARY_T[op](x)


def binary_t(a: Tensor, b: Tensor, op: str) -> Tensor:
    return _BINARY_T[op](a, b)


def conv_nd_t(x: Tensor, weight: Tensor, bias: Optional[Tensor], n: int, stride, padding, dilation,
              scale=None, shift=None, residual=None, act: int = 0, residual_first: bool = False,
              in_layout: int = 0, out_layout: int = 0, res_layout: int = 0) -> Tensor:
    if in_layout or out_layout or res_layout:
        raise RuntimeError("WideConv: gradients are available for the N-first layout only")
    nd = x.dim() - 3
    conv = (F.conv1d, F.conv2d, F.conv3d)[nd - 1]
    bsz, cin = x.shape[1], x.shape[2]
    y = conv(x.transpose(0, 1).reshape(bsz, n * cin, *x.shape[3:]), weight, bias, stride, padding, dilation, n)
    cout = weight.shape[0] // n
    y = y.reshape(bsz, n, cout, *y.shape[2:]).transpose(0, 1)
    if scale is not None:
        y = y * _chan_view(scale, n, cout, y.dim())
    if shift is not None:
        y = y + _chan_view(shift, n, cout, y.dim())
    if residual is not None and residual_first:
        y = y + residual
    y = act_t(y, act)
    if residual is not None and not residual_first:
        y = y + residual
    return y.contiguous()


def gru_t(x: Tensor, h0, w_ih: Tensor, w_hh: Tensor, b_ih, b_hh):
    n, b, t, _ = x.shape
    hsz = w_hh.shape[2]
    gx = linear_t(x, w_ih, b_ih)                                     # [N, B, T, 3H]
    h = h0 if h0 is not None else x.new_zeros(n, b, hsz)
    outs = []
    for s in range(t):
        gh = linear_t(h, w_hh, b_hh)                                 # [N, B, 3H]
        xr, xz, xn = gx[:, :, s].chunk(3, dim=-1)
        hr, hz, hn = gh.chunk(3, dim=-1)
        r = torch.sigmoid(xr + hr)
        z = torch.sigmoid(xz + hz)
        nn_ = torch.tanh(xn + r * hn)
        h = (1 - z) * nn_ + z * h
        outs.append(h)
    out = torch.stack(outs, dim=2) if outs else x.new_zeros(n, b, 0, hsz)
    return out, h


def lstm_t(x: Tensor, h0, c0, w_ih: Tensor, w_hh: Tensor, b_ih, b_hh):
    n, b, t, _ = x.shape
    hsz = w_hh.shape[2]
    gx = linear_t(x, w_ih, b_ih)                                     # [N, B, T, 4H]
    h = h0 if h0 is not None else x.new_zeros(n, b, hsz)
    c = c0 if c0 is not None else x.new_zeros(n, b, hsz)
    outs = []
    for s in range(t):
        g = gx[:, :, s] + linear_t(h, w_hh, b_hh)
        i, f, gg, o = g.chunk(4, dim=-1)
        c = torch.sigmoid(f) * c + torch.sigmoid(i) * torch.tanh(gg)
        h = torch.sigmoid(o) * torch.tanh(c)
        outs.append(h)
    out = torch.stack(outs, dim=2) if outs else x.new_zeros(n, b, 0, hsz)
    return out, h, c


def attention_t(query: Tensor, key: Tensor, value: Tensor, attn_mask, is_causal: bool, n_heads: int,
                q_weight: Tensor, q_bias, kv_weight: Tensor, kv_bias, out_weight: Tensor, out_bias) -> Tensor:
    n, b, tq, d = query.shape
    tk = key.shape[2]
    dh = d // n_heads
    q = linear_t(query, q_weight, q_bias)
    kb = None if kv_bias is None else kv_bias[:, :d]
    vb = None if kv_bias is None else kv_bias[:, d:]
    k = linear_t(key, kv_weight[:, :d], kb)
    v = linear_t(value, kv_weight[:, d:], vb)
    split = lambda t, tt: t.reshape(n * b, tt, n_heads, dh).transpose(1, 2)
    mask = attn_mask
    if mask is not None:
        mask = torch.broadcast_to(mask.to(query.device), (n * b, n_heads, tq, tk))
    o = F.scaled_dot_product_attention(split(q, tq), split(k, tk), split(v, tk), attn_mask=mask,
                                       is_causal=is_causal, scale=1.0 / math.sqrt(dh))
    o = o.transpose(1, 2).reshape(n, b, tq, d)
    return linear_t(o, out_weight, out_bias)


# ---------------------------------------------------------------------------
# Kernel-backed gradients
#
# WideLinear (with its fused ReLU / GELU), WideLayerNorm and the layout swap
# have backward kernels (csrc/backward.cu): their forward runs once, on the
# kernels, and the backward launches the gradient kernels on the saved
# tensors instead of re-running a torch formulation.
# ---------------------------------------------------------------------------
_KERNEL_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


class LinearFn(torch.autograd.Function):
    """y = act(x W^T + b) per model; backward: widek_act_bwd then
    widek_linear_bwd (dX, dW, db). ReLU keeps its output for the gradient;
    GELU runs unfused (GEMM, then the GELU kernel) and keeps its input."""

    @staticmethod
    def forward(ctx, x, weight, bias, act):
        from . import ops
        with torch.no_grad():
            if act == 2:
                pre = ops.linear(x, weight, bias, 0)
                y, saved = ops.unary(pre, 'gelu'), pre
            else:
                y = ops.linear(x, weight, bias, act)
                saved = y if act == 1 else None
        ctx.act, ctx.has_bias = act, bias is not None
        ctx.save_for_backward(x, weight, saved)
        return y

    @staticmethod
    def backward(ctx, dy):
        from . import ops
        x, weight, saved = ctx.saved_tensors
        dy = dy.to(weight.dtype).contiguous()
        if ctx.act:
            dy = ops.act_bwd(dy, saved, ctx.act)
        need_x, need_w, need_b = ctx.needs_input_grad[:3]
        dx, dw, db = ops.linear_bwd(x, weight, dy, need_x, need_w, need_b and ctx.has_bias)
        if dx is not None:
            dx = dx.view(x.shape)
        return dx, dw, db, None


class LayerNormFn(torch.autograd.Function):
    """LayerNorm with per-model affine; backward: widek_layernorm_bwd."""

    @staticmethod
    def forward(ctx, x, weight, bias, n, d, eps):
        from . import ops
        with torch.no_grad():
            y = ops.layernorm(x, weight, bias, n, d, eps)
        ctx.n, ctx.d, ctx.eps, ctx.bias_shape = n, d, eps, bias.shape
        ctx.save_for_backward(x, weight)
        return y

    @staticmethod
    def backward(ctx, dy):
        from . import ops
        x, weight = ctx.saved_tensors
        dx, dw, db = ops.layernorm_bwd(x, weight, dy.to(x.dtype).contiguous(), ctx.n, ctx.d, ctx.eps,
                                       ctx.needs_input_grad[1], ctx.needs_input_grad[2])
        dw = None if dw is None else dw.view(weight.shape)
        db = None if db is None else db.view(ctx.bias_shape)
        return dx.view(x.shape), dw, db, None, None, None


class Swap01Fn(torch.autograd.Function):
    """[A, B, ...] -> [B, A, ...]; its gradient is the same swap."""

    @staticmethod
    def forward(ctx, x):
        from . import ops
        with torch.no_grad():
            return ops.swap01(x)

    @staticmethod
    def backward(ctx, dy):
        from . import ops
        return ops.swap01(dy.contiguous())


class ActFn(torch.autograd.Function):
    """ReLU / GELU glue (traced_wide.py:174-186); backward: widek_act_bwd
    (ReLU from its output, GELU from its input)."""

    @staticmethod
    def forward(ctx, x, op):
        from . import ops
        with torch.no_grad():
            y = ops.unary(x, op)
        ctx.act = 1 if op == 'relu' else 2
        ctx.save_for_backward(y if op == 'relu' else x)
        return y

    @staticmethod
    def backward(ctx, dy):
        from . import ops
        saved, = ctx.saved_tensors
        return ops.act_bwd(dy.to(saved.dtype).contiguous(), saved, ctx.act).view(saved.shape), None


def unary_grad(x: Tensor, op: str) -> Tensor:
    from . import ops
    if op in ('relu', 'gelu') and x.is_cuda and x.dtype in _KERNEL_DTYPES:
        return ActFn.apply(x, op)
    return run(ops.unary, unary_t, x, op)


def linear_grad(x: Tensor, weight: Tensor, bias: Optional[Tensor], act: int) -> Tensor:
    """Differentiable WideLinear: the kernel-backed Function where the
    tensors fit it, else the recompute path."""
    from . import ops
    ok = (x.is_cuda and weight.dtype in _KERNEL_DTYPES and x.dtype == weight.dtype
          and (bias is None or bias.dtype == weight.dtype) and x.dim() >= 2 and weight.dim() == 3
          and x.shape[0] == weight.shape[0] and x.shape[-1] == weight.shape[2] and weight.shape[0] <= 65535)
    if not ok:
        return run(ops.linear, linear_t, x, weight, bias, act)
    return LinearFn.apply(x, weight, bias, act)


def layernorm_grad(x: Tensor, weight: Tensor, bias: Tensor, n: int, d: int, eps: float) -> Tensor:
    from . import ops
    ok = (x.is_cuda and x.dtype in _KERNEL_DTYPES and weight.dtype == x.dtype and bias.dtype == x.dtype
          and 0 < d <= 1024 and x.dim() >= 2 and x.shape[0] == n and x.shape[-1] == d and n <= 65535)
    if not ok:
        return run(ops.layernorm, layernorm_t, x, weight, bias, n, d, eps)
    return LayerNormFn.apply(x, weight, bias, n, d, eps)


class BatchNormFn(torch.autograd.Function):
    """BatchNorm on [N, B, C, *S] (batch or running statistics); backward:
    widek_batchnorm_bwd. Running statistics are updated once, in forward."""

    @staticmethod
    def forward(ctx, x, weight, bias, n, c, running_mean, running_var, use_batch_stats, update_running, momentum,
                eps):
        from . import ops
        with torch.no_grad():
            y = ops.batchnorm(x, n, c, weight, bias, running_mean, running_var, use_batch_stats, update_running,
                              momentum, eps)
        ctx.n, ctx.c, ctx.eps, ctx.batch_stats = n, c, eps, use_batch_stats
        ctx.has_w, ctx.has_b = weight is not None, bias is not None
        stats = (running_mean.clone(), running_var.clone()) if not use_batch_stats else (None, None)
        ctx.save_for_backward(x, weight, *stats)
        return y

    @staticmethod
    def backward(ctx, dy):
        from . import ops
        x, weight, rm, rv = ctx.saved_tensors
        dx, dw, db = ops.batchnorm_bwd(x, dy.to(x.dtype).contiguous(), ctx.n, ctx.c, weight, rm, rv, ctx.batch_stats,
                                       ctx.eps, ctx.needs_input_grad[1], ctx.needs_input_grad[2] and ctx.has_b)
        return (dx.view(x.shape), None if dw is None else dw.view(weight.shape), db, None, None, None, None, None,
                None, None, None)


class GroupNormFn(torch.autograd.Function):
    """GroupNorm on [N, B, C, *S] (also InstanceNorm); backward:
    widek_groupnorm_bwd."""

    @staticmethod
    def forward(ctx, x, weight, bias, n, groups, eps):
        from . import ops
        with torch.no_grad():
            y = ops.groupnorm(x, n, groups, weight, bias, eps)
        ctx.n, ctx.groups, ctx.eps, ctx.has_b = n, groups, eps, bias is not None
        ctx.bias_shape = None if bias is None else bias.shape
        ctx.save_for_backward(x, weight)
        return y

    @staticmethod
    def backward(ctx, dy):
        from . import ops
        x, weight = ctx.saved_tensors
        dx, dw, db = ops.groupnorm_bwd(x, dy.to(x.dtype).contiguous(), ctx.n, ctx.groups, weight, ctx.eps,
                                       ctx.needs_input_grad[1], ctx.needs_input_grad[2] and ctx.has_b)
        return (dx.view(x.shape), None if dw is None else dw.view(weight.shape),
                None if db is None else db.view(ctx.bias_shape), None, None, None)


def batchnorm_grad(x, n, c, weight, bias, running_mean, running_var, use_batch_stats, update_running, momentum,
                   eps):
    from . import ops
    ok = (x.is_cuda and x.dtype in _KERNEL_DTYPES and x.dim() >= 3 and all(
        t is None or t.dtype == x.dtype for t in (weight, bias, running_mean, running_var))
        and (use_batch_stats or (running_mean is not None and running_var is not None)))
    if not ok:
        return run(ops.batchnorm, batchnorm_t, x, n, c, weight, bias, running_mean, running_var, use_batch_stats,
                   update_running, momentum, eps)
    return BatchNormFn.apply(x, weight, bias, n, c, running_mean, running_var, use_batch_stats, update_running,
                             momentum, eps)


def groupnorm_grad(x, n, groups, weight, bias, eps):
    from . import ops
    ok = (x.is_cuda and x.dtype in _KERNEL_DTYPES and x.dim() >= 3 and x.shape[2] % groups == 0
          and all(t is None or t.dtype == x.dtype for t in (weight, bias)))
    if not ok:
        return run(ops.groupnorm, groupnorm_t, x, n, groups, weight, bias, eps, False)
    return GroupNormFn.apply(x, weight, bias, n, groups, eps)
