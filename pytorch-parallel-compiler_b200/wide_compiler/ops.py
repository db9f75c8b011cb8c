"""Tensor-level wrappers over the libwidek C-ABI.

Each function validates its tensors (CUDA, one device, supported dtype),
makes them dense, allocates the output with torch's caching allocator, and
launches the kernel on torch's current stream. These are the only places the
wide primitives reach device code; nothing here computes on the host.
"""
from __future__ import annotations

import contextlib
import math
from typing import List, Optional, Sequence

import ctypes
import torch
from torch import Tensor

from . import _autograd as _AG
from . import _derived
from . import _native as N

ACT_NONE, ACT_RELU, ACT_GELU = N.ACT_NONE, N.ACT_RELU, N.ACT_GELU

UNARY_CODES = {"relu": 0, "gelu": 1, "sigmoid": 2, "tanh": 3, "silu": 4}
BINARY_CODES = {"add": 0, "mul": 1, "sub": 2, "div": 3}


def _compiling() -> bool:
    """Dynamo is tracing: the wide ops go through their torch.library
    operators (``_torch_ops``), which it can trace, instead of the ctypes
    calls, which it cannot."""
    return torch.compiler.is_compiling()


def _guard(dev: torch.device):
    if dev.index is None or dev.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(dev)


def _dense(t: Tensor) -> Tensor:
    return t if t.is_contiguous() else t.contiguous()


def _same_dtype(what: str, ref: Tensor, *others: Optional[Tensor]) -> None:
    for o in others:
        if o is not None and o.dtype != ref.dtype:
            raise TypeError(f"{what}: dtype mismatch ({ref.dtype} vs {o.dtype})")


# ---------------------------------------------------------------------------
# WideLinear
# ---------------------------------------------------------------------------

def linear(x: Tensor, weight: Tensor, bias: Optional[Tensor], act: int = ACT_NONE,
           force_simt: bool = False) -> Tensor:
    """y[i] = act(x[i] @ weight[i]^T + bias[i]).

    x: [N, ..., K] (any batch dims), weight: [N, O, K], bias: [N, O] or None.
    Returns [N, ..., O].
    """
    if _compiling() and not force_simt:
        return torch.ops.widek.linear(x, weight, bias, act)
    if _AG.needs_grad(x, weight, bias):
        if force_simt:
            return _AG.run(linear, _AG.linear_t, x, weight, bias, act, force_simt)
        return _AG.linear_grad(x, weight, bias, act)
    dev = N.require_cuda(x, weight, bias, what="WideLinear")
    _same_dtype("WideLinear", weight, x, bias)
    n, o, k = weight.shape
    if x.shape[0] != n or x.shape[-1] != k:
        raise ValueError(f"WideLinear: input {tuple(x.shape)} does not match weight {tuple(weight.shape)}")
    batch = x.shape[1:-1]
    xd = _dense(x)
    m = math.prod(batch)
    wd = _dense(weight)
    bd = _dense(bias) if bias is not None else None
    y = torch.empty((n, *batch, o), device=dev, dtype=weight.dtype)
    fn = N.lib().widek_linear_fwd_simt if force_simt else N.lib().widek_linear_fwd
    with _guard(dev):
        rc = fn(xd.data_ptr(), wd.data_ptr(), N.ptr(bd), y.data_ptr(), n, m, k, o,
                N.dtype_code(weight), act, N.stream_ptr(dev))
    N.check(rc, "widek_linear_fwd")
    return y


def transpose(x: Tensor) -> Tensor:
    """[batch, R, C] -> [batch, C, R] as one dense copy (widek_transpose)."""
    dev = N.require_cuda(x, what="transpose")
    if x.dim() != 3:
        raise ValueError(f"transpose: expected [batch, R, C], got {tuple(x.shape)}")
    xd = _dense(x)
    y = torch.empty((xd.shape[0], xd.shape[2], xd.shape[1]), device=dev, dtype=x.dtype)
    with _guard(dev):
        rc = N.lib().widek_transpose(xd.data_ptr(), y.data_ptr(), xd.shape[0], xd.shape[1], xd.shape[2],
                                     N.dtype_code(x), N.stream_ptr(dev))
    N.check(rc, "widek_transpose")
    return y


def linear_bwd(x: Tensor, weight: Tensor, dy: Tensor, need_dx: bool = True, need_dw: bool = True,
               need_db: bool = True):
    """Gradients of y = x W^T + b per model (no activation): (dx, dw, db),
    None where not asked. x [N, ..., K], weight [N, O, K], dy [N, ..., O]
    (widek_linear_bwd; the products on the forward's grouped GEMM)."""
    dev = N.require_cuda(x, weight, dy, what="WideLinear backward")
    _same_dtype("WideLinear backward", weight, x, dy)
    n, o, k = weight.shape
    m = math.prod(x.shape[1:-1])
    xd, wd, dyd = _dense(x), _dense(weight), _dense(dy)
    dx = torch.empty_like(xd) if need_dx else None
    dw = torch.empty_like(wd) if need_dw else None
    db = torch.empty((n, o), device=dev, dtype=weight.dtype) if need_db else None
    if not (need_dx or need_dw or need_db):
        return None, None, None
    code = N.dtype_code(weight)
    ws_bytes = N.lib().widek_linear_bwd_workspace(n, m, k, o, code)
    if ws_bytes < 0:
        raise ValueError(f"WideLinear backward: bad sizes n={n} m={m} k={k} o={o}")
    ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
    with _guard(dev):
        rc = N.lib().widek_linear_bwd(xd.data_ptr(), wd.data_ptr(), dyd.data_ptr(), N.ptr(dx), N.ptr(dw), N.ptr(db),
                                      n, m, k, o, code, ws.data_ptr(), ws_bytes, N.stream_ptr(dev))
    N.check(rc, "widek_linear_bwd")
    return dx, dw, db


def act_bwd(dy: Tensor, saved: Tensor, act: int) -> Tensor:
    """dy * act'(saved): ReLU from its output, GELU (erf) from its input."""
    dev = N.require_cuda(dy, saved, what="activation backward")
    _same_dtype("activation backward", dy, saved)
    if dy.shape != saved.shape:
        raise ValueError(f"activation backward: {tuple(dy.shape)} vs {tuple(saved.shape)}")
    dyd, sd = _dense(dy), _dense(saved)
    out = torch.empty_like(dyd)
    with _guard(dev):
        rc = N.lib().widek_act_bwd(dyd.data_ptr(), sd.data_ptr(), out.data_ptr(), dyd.numel(), act,
                                   N.dtype_code(dy), N.stream_ptr(dev))
    N.check(rc, "widek_act_bwd")
    return out


def linear_layout(x: Tensor, weight: Tensor, bias: Optional[Tensor], act: int, in_packed: bool,
                  out_packed: bool) -> Tensor:
    """WideLinear with the packed boundary layout on either side: x is
    [B, N*T, K] when ``in_packed`` (else N-first [N, B, T, K]), the result
    [B, N*T, O] when ``out_packed`` (else [N, B, T, O]). The kernels read and
    write the packed rows in place (widek_linear_fwd_ex); equal to unpacking,
    ``linear`` and packing (traced_wide.py:463-469, :527-532)."""
    dev = N.require_cuda(x, weight, bias, what="WideLinear")
    _same_dtype("WideLinear", weight, x, bias)
    n, o, k = weight.shape
    if x.dim() != (3 if in_packed else 4) or x.shape[-1] != k or (in_packed and x.shape[1] % n != 0) \
            or (not in_packed and x.shape[0] != n):
        raise ValueError(f"WideLinear: input {tuple(x.shape)} does not match weight {tuple(weight.shape)} "
                         f"({'packed' if in_packed else 'N-first'})")
    b, t = (x.shape[0], x.shape[1] // n) if in_packed else (x.shape[1], x.shape[2])
    y = torch.empty((b, n * t, o) if out_packed else (n, b, t, o), device=dev, dtype=weight.dtype)
    xd, wd = _dense(x), _dense(weight)
    bd = _dense(bias) if bias is not None else None
    with _guard(dev):
        rc = N.lib().widek_linear_fwd_ex(xd.data_ptr(), wd.data_ptr(), N.ptr(bd), y.data_ptr(), n, b * t, k, o, t,
                                         LAYOUT_PACKED if in_packed else LAYOUT_NFIRST,
                                         LAYOUT_PACKED if out_packed else LAYOUT_NFIRST, N.dtype_code(weight), act,
                                         N.stream_ptr(dev))
    N.check(rc, "widek_linear_fwd_ex")
    return y


def linear_ln_layout(x: Tensor, weight: Tensor, bias: Optional[Tensor], ln_weight: Tensor, ln_bias: Tensor,
                     eps: float, in_packed: bool, out_packed: bool) -> Optional[Tensor]:
    """LayerNorm(x @ weight^T + bias) with the per-model affine (ln_weight /
    ln_bias flat [N*O]) in one launch (widek_linear_ln_fwd_ex): the attention
    output projection (wide_attention.py:233-236) followed by WideLayerNorm
    (wide_layernorm.py:62-65). Layouts as ``linear_layout``; None, launching
    nothing, when the kernel does not take the shapes (the caller runs the
    two ops)."""
    dev = N.require_cuda(x, weight, bias, ln_weight, ln_bias, what="WideLinear + LayerNorm")
    _same_dtype("WideLinear + LayerNorm", weight, x, bias, ln_weight, ln_bias)
    n, o, k = weight.shape
    if x.dim() != (3 if in_packed else 4) or x.shape[-1] != k or (in_packed and x.shape[1] % n != 0) \
            or (not in_packed and x.shape[0] != n) or ln_weight.numel() != n * o or ln_bias.numel() != n * o:
        return None
    b, t = (x.shape[0], x.shape[1] // n) if in_packed else (x.shape[1], x.shape[2])
    y = torch.empty((b, n * t, o) if out_packed else (n, b, t, o), device=dev, dtype=weight.dtype)
    xd, wd = _dense(x), _dense(weight)
    bd = _dense(bias) if bias is not None else None
    with _guard(dev):
        rc = N.lib().widek_linear_ln_fwd_ex(xd.data_ptr(), wd.data_ptr(), N.ptr(bd), _dense(ln_weight).data_ptr(),
                                            _dense(ln_bias).data_ptr(), y.data_ptr(), n, b * t, k, o, t,
                                            LAYOUT_PACKED if in_packed else LAYOUT_NFIRST,
                                            LAYOUT_PACKED if out_packed else LAYOUT_NFIRST, float(eps),
                                            N.dtype_code(weight), N.stream_ptr(dev))
    if rc == N.WIDEK_ERR_UNSUPPORTED:
        return None
    N.check(rc, "widek_linear_ln_fwd_ex")
    return y


_CHAIN_MEMO: dict = {}


def mlp_chain(x: Tensor, weights: Sequence[Tensor], biases: Sequence[Optional[Tensor]], acts: Sequence[int],
              n: int, in_layout: int = 0, out_layout: int = 0) -> Optional[Tensor]:
    """A chain of wide Linears with activations in one launch:
    h = act_l(h @ weights[l][i]^T + biases[l][i]) per model i.

    weights[l]: [N, D_{l+1}, D_l]; x: [N, B, D_0] (in_layout 0, N-first) or
    [B, N*D_0] (in_layout 1, packed); the result is [N, B, D_L] or
    [B, N*D_L] per out_layout. Returns None, launching nothing, when the
    chain does not fit the one-CTA-per-model kernel. The argument arrays and
    the fit query are memoised per (pointers, shapes, layouts, dtype)."""
    if _AG.needs_grad(x, weights, biases):
        # training: layer by layer, each WideLinear with its backward kernels
        if not 1 <= len(weights) <= 8 or len(biases) != len(weights) or len(acts) != len(weights):
            return None
        h = swap01(x.reshape(x.shape[0], n, -1)) if in_layout == 1 else x
        for w, b, a in zip(weights, biases, acts):
            h = linear(h, w, b, a)
        return swap01(h).reshape(h.shape[1], -1) if out_layout == 1 else h
    layers = len(weights)
    if not 1 <= layers <= 8 or len(biases) != layers or len(acts) != layers:
        return None
    wd = [w if w.is_contiguous() else w.contiguous() for w in weights]
    bd = [b if b is None or b.is_contiguous() else b.contiguous() for b in biases]
    batch = x.shape[0] if in_layout == 1 else (x.shape[1] if x.dim() == 3 else -1)
    key = (tuple(w.data_ptr() for w in wd), tuple(0 if b is None else b.data_ptr() for b in bd),
           tuple(tuple(w.shape) for w in wd), tuple(acts), n, batch, tuple(x.shape), in_layout, out_layout,
           x.dtype, x.device)
    plan = _CHAIN_MEMO.get(key)
    if plan is None:
        dev = N.require_cuda(x, *weights, *biases, what="WideLinear chain")
        _same_dtype("WideLinear chain", weights[0], x, *weights, *biases)
        dims = [weights[0].shape[2]] + [w.shape[1] for w in weights]
        for l, w in enumerate(weights):
            if w.dim() != 3 or w.shape[0] != n or w.shape[2] != dims[l]:
                raise ValueError(f"WideLinear chain: weight {l} {tuple(w.shape)} does not follow width {dims[l]}")
            b = biases[l]
            if b is not None and tuple(b.shape) != (n, dims[l + 1]):
                raise ValueError(f"WideLinear chain: bias {l} {tuple(b.shape)} is not [{n}, {dims[l + 1]}]")
        if in_layout == 1:
            if x.dim() != 2 or x.shape[1] != n * dims[0]:
                raise ValueError(f"WideLinear chain: packed input {tuple(x.shape)} is not [B, {n}*{dims[0]}]")
        elif x.dim() != 3 or x.shape[0] != n or x.shape[2] != dims[0]:
            raise ValueError(f"WideLinear chain: input {tuple(x.shape)} is not [{n}, B, {dims[0]}]")
        c_dims = (ctypes.c_int64 * (layers + 1))(*dims)
        c_acts = (ctypes.c_int * layers)(*acts)
        code = N.dtype_code(x)
        ok = bool(N.lib().widek_mlp_chain_supported(c_dims, c_acts, layers, n, batch, code))
        c_w = (ctypes.c_void_p * layers)(*[w.data_ptr() for w in wd])
        c_b = (ctypes.c_void_p * layers)(*[N.ptr(b) for b in bd])
        out_shape = (batch, n * dims[-1]) if out_layout == 1 else (n, batch, dims[-1])
        plan = (ok, c_dims, c_acts, c_w, c_b, code, out_shape, dev)
        if len(_CHAIN_MEMO) > 256:
            _CHAIN_MEMO.clear()
        _CHAIN_MEMO[key] = plan
    ok, c_dims, c_acts, c_w, c_b, code, out_shape, dev = plan
    if not ok:
        return None
    xd = x if x.is_contiguous() else x.contiguous()
    y = torch.empty(out_shape, device=dev, dtype=x.dtype)
    with _guard(dev):
        rc = N.lib().widek_mlp_chain_fwd(xd.data_ptr(), y.data_ptr(), c_w, c_b, c_dims, c_acts, layers, n, batch,
                                         in_layout, out_layout, code, N.stream_ptr(dev))
    N.check(rc, "widek_mlp_chain_fwd")
    return y


# ---------------------------------------------------------------------------
# WideLayerNorm
# ---------------------------------------------------------------------------

def layernorm(x: Tensor, weight: Tensor, bias: Tensor, n: int, d: int, eps: float) -> Tensor:
    """LayerNorm over the last dim with per-model affine (weight/bias flat [n*d])."""
    if _compiling():
        return torch.ops.widek.layernorm(x, weight, bias, n, d, eps)
    if _AG.needs_grad(x, weight, bias):
        return _AG.layernorm_grad(x, weight, bias, n, d, eps)
    dev = N.require_cuda(x, weight, bias, what="WideLayerNorm")
    _same_dtype("WideLayerNorm", x, weight, bias)
    if x.shape[0] != n or x.shape[-1] != d:
        raise ValueError(f"WideLayerNorm: input {tuple(x.shape)} is not [N={n}, ..., D={d}]")
    xd = _dense(x)
    rows = xd.numel() // (n * d) if n * d > 0 else 0
    y = torch.empty_like(xd)
    with _guard(dev):
        rc = N.lib().widek_layernorm_fwd(xd.data_ptr(), _dense(weight).data_ptr(), _dense(bias).data_ptr(),
                                         y.data_ptr(), n, rows, d, float(eps), N.dtype_code(x),
                                         N.stream_ptr(dev))
    N.check(rc, "widek_layernorm_fwd")
    return y


def layernorm_bwd(x: Tensor, weight: Tensor, dy: Tensor, n: int, d: int, eps: float, need_dw: bool = True,
                  need_db: bool = True):
    """Gradients of the per-model LayerNorm: (dx, dweight, dbias), None where
    not asked (widek_layernorm_bwd; statistics recomputed from x)."""
    dev = N.require_cuda(x, weight, dy, what="WideLayerNorm backward")
    _same_dtype("WideLayerNorm backward", x, weight, dy)
    xd, wd, dyd = _dense(x), _dense(weight), _dense(dy)
    outer = xd.numel() // (n * d) if n * d > 0 else 0
    dx = torch.empty_like(xd)
    dw = torch.empty((n * d,), device=dev, dtype=weight.dtype) if need_dw else None
    db = torch.empty((n * d,), device=dev, dtype=weight.dtype) if need_db else None
    ws_bytes = N.lib().widek_layernorm_bwd_workspace(n, outer, d)
    if ws_bytes < 0:
        raise ValueError(f"WideLayerNorm backward: bad sizes n={n} rows={outer} d={d}")
    ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
    with _guard(dev):
        rc = N.lib().widek_layernorm_bwd(xd.data_ptr(), wd.data_ptr(), dyd.data_ptr(), dx.data_ptr(), N.ptr(dw),
                                         N.ptr(db), n, outer, d, float(eps), N.dtype_code(x), ws.data_ptr(),
                                         ws_bytes, N.stream_ptr(dev))
    N.check(rc, "widek_layernorm_bwd")
    return dx, dw, db


def layernorm_packed(x: Tensor, weight: Tensor, bias: Tensor, n: int, d: int, eps: float) -> Tensor:
    """LayerNorm of N models on the packed boundary layout: x [B, N*T, ..., D]
    (or [B, N*D]) -> same layout, model i's affine applied to its rows
    (widek_layernorm_fwd_ex, outer = B). Equals packing the LayerNorm of the
    unpacked N-first tensor (traced_wide.py:463-469, :527-532)."""
    dev = N.require_cuda(x, weight, bias, what="WideLayerNorm")
    _same_dtype("WideLayerNorm", x, weight, bias)
    if x.dim() == 2:
        ok = x.shape[1] == n * d
    else:
        ok = x.dim() > 2 and x.shape[-1] == d and x.shape[1] % n == 0
    if not ok:
        raise ValueError(f"WideLayerNorm: packed input {tuple(x.shape)} does not hold N={n} models of D={d}")
    xd = _dense(x)
    outer = xd.shape[0]
    inner = xd.numel() // (outer * n * d) if outer * n * d > 0 else 0
    y = torch.empty_like(xd)
    with _guard(dev):
        rc = N.lib().widek_layernorm_fwd_ex(xd.data_ptr(), _dense(weight).data_ptr(), _dense(bias).data_ptr(),
                                            y.data_ptr(), n, outer, inner, d, float(eps), N.dtype_code(x),
                                            N.stream_ptr(dev))
    N.check(rc, "widek_layernorm_fwd_ex")
    return y


# ---------------------------------------------------------------------------
# Layout boundary
# ---------------------------------------------------------------------------

def swap01(x: Tensor) -> Tensor:
    """[A, B, *rest] -> [B, A, *rest] as one dense copy (rows of prod(rest))."""
    if _compiling():
        return torch.ops.widek.swap01(x)
    if _AG.needs_grad(x):
        return _AG.Swap01Fn.apply(x)
    dev = N.require_cuda(x, what="swap01")
    xd = _dense(x)
    a, b = xd.shape[0], xd.shape[1]
    rest = xd.shape[2:]
    y = torch.empty((b, a, *rest), device=dev, dtype=x.dtype)
    inner = xd.numel() // max(1, a * b) * xd.element_size() if a * b > 0 else 0
    with _guard(dev):
        rc = N.lib().widek_swap01(xd.data_ptr(), y.data_ptr(), a, b, inner, N.stream_ptr(dev))
    N.check(rc, "widek_swap01")
    return y


def pack(inputs: Sequence[Tensor]) -> Tensor:
    """Stacks N tensors [B, *F] into [B, N, *F] (one kernel, N source pointers)."""
    if _AG.needs_grad(list(inputs)):
        return _AG.run(pack, _AG.pack_t, list(inputs))
    dev = N.require_cuda(*inputs, what="pack")
    t0 = inputs[0]
    for t in inputs[1:]:
        if t.shape != t0.shape or t.dtype != t0.dtype:
            raise ValueError("pack: all inputs must share shape and dtype")
    dense = [_dense(t) for t in inputs]
    b = t0.shape[0]
    n = len(dense)
    out = torch.empty((b, n, *t0.shape[1:]), device=dev, dtype=t0.dtype)
    inner = (t0.numel() // b) * t0.element_size() if b > 0 else 0
    arr = (ctypes.c_void_p * n)(*[t.data_ptr() for t in dense])
    with _guard(dev):
        rc = N.lib().widek_pack(arr, n, out.data_ptr(), b, inner, N.stream_ptr(dev))
    N.check(rc, "widek_pack")
    return out


# ---------------------------------------------------------------------------
# Elementwise glue
# ---------------------------------------------------------------------------

def unary(x: Tensor, op: str) -> Tensor:
    if _compiling():
        return torch.ops.widek.unary(x, op)
    if _AG.needs_grad(x):
        return _AG.unary_grad(x, op)
    dev = N.require_cuda(x, what=f"unary {op}")
    xd = _dense(x)
    y = torch.empty_like(xd)
    with _guard(dev):
        rc = N.lib().widek_unary(xd.data_ptr(), y.data_ptr(), xd.numel(), UNARY_CODES[op], N.dtype_code(x),
                                 N.stream_ptr(dev))
    N.check(rc, f"widek_unary({op})")
    return y


def binary(a: Tensor, b: Tensor, op: str) -> Tensor:
    if _compiling():
        return torch.ops.widek.binary(a, b, op)
    if _AG.needs_grad(a, b):
        return _AG.run(binary, _AG.binary_t, a, b, op)
    dev = N.require_cuda(a, b, what=f"binary {op}")
    _same_dtype(f"binary {op}", a, b)
    if a.shape != b.shape:
        raise ValueError(f"binary {op}: shapes differ ({tuple(a.shape)} vs {tuple(b.shape)})")
    ad, bd = _dense(a), _dense(b)
    y = torch.empty_like(ad)
    with _guard(dev):
        rc = N.lib().widek_binary(ad.data_ptr(), bd.data_ptr(), y.data_ptr(), ad.numel(), BINARY_CODES[op],
                                  N.dtype_code(a), N.stream_ptr(dev))
    N.check(rc, f"widek_binary({op})")
    return y


# ---------------------------------------------------------------------------
# Norms
# ---------------------------------------------------------------------------

def _nbcl(x: Tensor, n: int, c: int, what: str):
    if x.dim() < 3 or x.shape[0] != n or x.shape[2] != c:
        raise ValueError(f"{what}: input {tuple(x.shape)} is not [N={n}, B, C={c}, ...]")
    return x.shape[1], math.prod(x.shape[3:])


def batchnorm(x: Tensor, n: int, c: int, weight: Optional[Tensor], bias: Optional[Tensor],
              running_mean: Optional[Tensor], running_var: Optional[Tensor], use_batch_stats: bool,
              update_running: bool, momentum: float, eps: float) -> Tensor:
    """Per-(model, channel) batch normalization on [N, B, C, *S]; weight, bias
    and running stats flat [N*C]. With use_batch_stats the running stats (if
    update_running) are updated in place."""
    if _compiling():
        return torch.ops.widek.batchnorm(x, n, c, weight, bias, running_mean, running_var, use_batch_stats,
                                         update_running, momentum, eps)
    if _AG.needs_grad(x, weight, bias):
        return _AG.batchnorm_grad(x, n, c, weight, bias, running_mean, running_var, use_batch_stats,
                                  update_running, momentum, eps)
    dev = N.require_cuda(x, weight, bias, running_mean, running_var, what="WideBatchNorm")
    _same_dtype("WideBatchNorm", x, weight, bias, running_mean, running_var)
    batch, l = _nbcl(x, n, c, "WideBatchNorm")
    xd = _dense(x)
    y = torch.empty_like(xd)
    code = N.dtype_code(x)
    with _guard(dev):
        if not use_batch_stats:
            if running_mean is None or running_var is None:
                raise ValueError("WideBatchNorm: eval mode needs running statistics")
            rc = N.lib().widek_batchnorm_fwd(xd.data_ptr(), y.data_ptr(), N.ptr(weight), N.ptr(bias),
                                             running_mean.data_ptr(), running_var.data_ptr(), n, batch, c, l,
                                             float(eps), code, N.stream_ptr(dev))
            N.check(rc, "widek_batchnorm_fwd")
            return y
        ws_bytes = N.lib().widek_batchnorm_train_workspace(n, batch, c, l)
        ws = torch.empty(max(int(ws_bytes), 16), dtype=torch.uint8, device=dev)
        rm = running_mean if update_running else None
        rv = running_var if update_running else None
        rc = N.lib().widek_batchnorm_train_fwd(xd.data_ptr(), y.data_ptr(), N.ptr(weight), N.ptr(bias), N.ptr(rm),
                                               N.ptr(rv), None, None, ws.data_ptr(), ws.numel(), n, batch, c, l,
                                               float(momentum), float(eps), code, N.stream_ptr(dev))
    N.check(rc, "widek_batchnorm_train_fwd")
    return y


def batchnorm_bwd(x: Tensor, dy: Tensor, n: int, c: int, weight: Optional[Tensor], running_mean: Optional[Tensor],
                  running_var: Optional[Tensor], batch_stats: bool, eps: float, need_dw: bool = True,
                  need_db: bool = True):
    """Gradients of ``batchnorm``: (dx, dweight, dbias), None where not asked
    or without affine parameters (widek_batchnorm_bwd)."""
    dev = N.require_cuda(x, dy, weight, running_mean, running_var, what="WideBatchNorm backward")
    _same_dtype("WideBatchNorm backward", x, dy, weight, running_mean, running_var)
    batch, l = _nbcl(x, n, c, "WideBatchNorm backward")
    xd, dyd = _dense(x), _dense(dy)
    dx = torch.empty_like(xd)
    dw = torch.empty((n * c,), device=dev, dtype=x.dtype) if need_dw and weight is not None else None
    db = torch.empty((n * c,), device=dev, dtype=x.dtype) if need_db else None
    with _guard(dev):
        rc = N.lib().widek_batchnorm_bwd(xd.data_ptr(), dyd.data_ptr(), N.ptr(_opt_dense(weight)),
                                         N.ptr(_opt_dense(running_mean)), N.ptr(_opt_dense(running_var)),
                                         dx.data_ptr(), N.ptr(dw), N.ptr(db), n, batch, c, l, int(batch_stats),
                                         float(eps), N.dtype_code(x), N.stream_ptr(dev))
    N.check(rc, "widek_batchnorm_bwd")
    return dx, dw, db


def groupnorm_bwd(x: Tensor, dy: Tensor, n: int, groups: int, weight: Optional[Tensor], eps: float,
                  need_dw: bool = True, need_db: bool = True):
    """Gradients of ``groupnorm``: (dx, dweight, dbias), None where not asked
    (widek_groupnorm_bwd; statistics recomputed from x)."""
    dev = N.require_cuda(x, dy, weight, what="WideGroupNorm backward")
    _same_dtype("WideGroupNorm backward", x, dy, weight)
    batch, c = x.shape[1], x.shape[2]
    l = math.prod(x.shape[3:])
    xd, dyd = _dense(x), _dense(dy)
    dx = torch.empty_like(xd)
    dw = torch.empty((n * c,), device=dev, dtype=x.dtype) if need_dw and weight is not None else None
    db = torch.empty((n * c,), device=dev, dtype=x.dtype) if need_db else None
    ws_bytes = N.lib().widek_groupnorm_bwd_workspace(n, batch, c)
    ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
    with _guard(dev):
        rc = N.lib().widek_groupnorm_bwd(xd.data_ptr(), dyd.data_ptr(), N.ptr(_opt_dense(weight)), dx.data_ptr(),
                                         N.ptr(dw), N.ptr(db), n, batch, c, l, groups, float(eps), N.dtype_code(x),
                                         ws.data_ptr(), ws_bytes, N.stream_ptr(dev))
    N.check(rc, "widek_groupnorm_bwd")
    return dx, dw, db


def groupnorm(x: Tensor, n: int, groups: int, weight: Optional[Tensor], bias: Optional[Tensor], eps: float,
              row_stats: bool = False):
    """GroupNorm on [N, B, C, *S] with statistics per (model, sample, group).
    With row_stats also returns fp32 (mean, biased var) of shape [N, B, groups]."""
    if _compiling() and not row_stats:
        return torch.ops.widek.groupnorm(x, n, groups, weight, bias, eps)
    if _AG.needs_grad(x, weight, bias):
        if row_stats:
            return _AG.run(groupnorm, _AG.groupnorm_t, x, n, groups, weight, bias, eps, row_stats)
        return _AG.groupnorm_grad(x, n, groups, weight, bias, eps)
    dev = N.require_cuda(x, weight, bias, what="WideGroupNorm")
    _same_dtype("WideGroupNorm", x, weight, bias)
    if x.dim() < 3 or x.shape[0] != n:
        raise ValueError(f"WideGroupNorm: input {tuple(x.shape)} is not [N={n}, B, C, ...]")
    batch, c = x.shape[1], x.shape[2]
    l = math.prod(x.shape[3:])
    xd = _dense(x)
    y = torch.empty_like(xd)
    mean = var = None
    if row_stats:
        mean = torch.empty(n, batch, groups, device=dev, dtype=torch.float32)
        var = torch.empty_like(mean)
    with _guard(dev):
        rc = N.lib().widek_groupnorm_fwd(xd.data_ptr(), y.data_ptr(), N.ptr(weight), N.ptr(bias), N.ptr(mean),
                                         N.ptr(var), n, batch, c, l, groups, float(eps), N.dtype_code(x),
                                         N.stream_ptr(dev))
    N.check(rc, "widek_groupnorm_fwd")
    return (y, mean, var) if row_stats else y


def instancenorm_train(x: Tensor, n: int, c: int, weight: Optional[Tensor], bias: Optional[Tensor],
                       running_mean: Tensor, running_var: Tensor, momentum: float, eps: float) -> Tensor:
    """InstanceNorm in training mode with tracked running stats: instance
    statistics for the output; running stats move toward the batch average of
    the instance mean / unbiased variance (torch.nn.InstanceNorm semantics)."""
    y, mean, var = groupnorm(x, n, c, weight, bias, eps, row_stats=True)
    l = math.prod(x.shape[3:])
    unbiased = var * (l / max(l - 1, 1))
    with torch.no_grad():
        running_mean.mul_(1 - momentum).add_(mean.mean(dim=1).reshape(-1).to(running_mean.dtype), alpha=momentum)
        running_var.mul_(1 - momentum).add_(unbiased.mean(dim=1).reshape(-1).to(running_var.dtype), alpha=momentum)
    return y


# ---------------------------------------------------------------------------
# Embedding
# ---------------------------------------------------------------------------

def embedding(idx: Tensor, weight: Tensor) -> Tensor:
    """[N, V, D] tables, shared integer indices of any shape -> [N, *idx.shape, D]."""
    if _compiling():
        return torch.ops.widek.embedding(idx, weight)
    if _AG.needs_grad(weight):
        return _AG.run(embedding, _AG.embedding_t, idx, weight)
    dev = N.require_cuda(idx, weight, what="WideEmbedding")
    if idx.dtype not in (torch.int64, torch.int32, torch.int16, torch.int8, torch.uint8):
        raise TypeError(f"WideEmbedding: indices must be integers, got {idx.dtype}")
    ii = _dense(idx.to(torch.int64))
    n, v, d = weight.shape
    wd = _dense(weight)
    out = torch.empty((n, *idx.shape, d), device=dev, dtype=weight.dtype)
    with _guard(dev):
        rc = N.lib().widek_embedding_fwd(ii.data_ptr(), wd.data_ptr(), out.data_ptr(), n, ii.numel(), v, d,
                                         N.dtype_code(weight), N.stream_ptr(dev))
    N.check(rc, "widek_embedding_fwd")
    return out


# ---------------------------------------------------------------------------
# Recurrent layers
# ---------------------------------------------------------------------------

def _rnn_check(x: Tensor, w_ih: Tensor, w_hh: Tensor, gates: int, what: str):
    if x.dim() != 4:
        raise ValueError(f"{what}: input must be [N, B, T, I], got {tuple(x.shape)}")
    n, batch, steps, i = x.shape
    if w_ih.dim() != 3 or w_ih.shape[0] != n or w_ih.shape[2] != i:
        raise ValueError(f"{what}: weight_ih {tuple(w_ih.shape)} does not match input {tuple(x.shape)}")
    hidden = w_hh.shape[2]
    if w_hh.shape != (n, gates * hidden, hidden) or w_ih.shape[1] != gates * hidden:
        raise ValueError(f"{what}: weight_hh {tuple(w_hh.shape)} is not [N, {gates}H, H]")
    return n, batch, steps, hidden


def _rnn_fwd(lstm: bool, x: Tensor, h0, c0, w_ih: Tensor, w_hh: Tensor, b_ih, b_hh, strides, n: int, hidden: int,
             packed: bool = False):
    """One library call for the whole forward: the input projection (reading
    W_ih by (model, row) strides, into a workspace) and the recurrence
    (W_hh by strides). With ``packed`` x is the boundary layout
    [B, N*T, I] and out is written as [B, N*T, H]."""
    dev = x.device
    if packed:
        batch, steps, inp = x.shape[0], x.shape[1] // n, x.shape[2]
        out = torch.empty(batch, n * steps, hidden, device=dev, dtype=x.dtype)
    else:
        _, batch, steps, inp = x.shape
        out = torch.empty(n, batch, steps, hidden, device=dev, dtype=x.dtype)
    lay = LAYOUT_PACKED if packed else LAYOUT_NFIRST
    hn = torch.empty(n, batch, hidden, device=dev, dtype=x.dtype)
    cn = torch.empty(n, batch, hidden, device=dev, dtype=x.dtype) if lstm else None
    code = N.dtype_code(x)
    ws_bytes = int(N.lib().widek_rnn_workspace(1 if lstm else 0, n, batch, steps, hidden, code))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    c_strides = (ctypes.c_int64 * 4)(*strides)
    xd = _dense(x)
    with _guard(dev):
        if lstm:
            rc = N.lib().widek_lstm_fwd_ex(xd.data_ptr(), w_ih.data_ptr(), w_hh.data_ptr(), N.ptr(b_ih),
                                           N.ptr(b_hh), N.ptr(h0), N.ptr(c0), out.data_ptr(), hn.data_ptr(),
                                           cn.data_ptr(), c_strides, ws.data_ptr(), ws.numel(), n, batch, steps, inp,
                                           hidden, lay, lay, code, N.stream_ptr(dev))
        else:
            rc = N.lib().widek_gru_fwd_ex(xd.data_ptr(), w_ih.data_ptr(), w_hh.data_ptr(), N.ptr(b_ih), N.ptr(b_hh),
                                          N.ptr(h0), out.data_ptr(), hn.data_ptr(), c_strides, ws.data_ptr(),
                                          ws.numel(), n, batch, steps, inp, hidden, lay, lay, code,
                                          N.stream_ptr(dev))
    N.check(rc, "widek_lstm_fwd_ex" if lstm else "widek_gru_fwd_ex")
    return out, hn, cn


def _packed_rnn_check(x: Tensor, n: int, what: str) -> None:
    if x.dim() != 3 or x.shape[1] % n != 0:
        raise ValueError(f"{what}: packed input must be [B, N*T, I] with N={n}, got {tuple(x.shape)}")


def gru_packed(x: Tensor, w_ih: Tensor, w_hh: Tensor, b_ih: Optional[Tensor], b_hh: Optional[Tensor]):
    """WideGRU forward on the packed boundary layout, zero initial state:
    x [B, N*T, I] -> (out [B, N*T, H] packed, h_n [N, B, H]), equal to
    packing the output of ``gru`` on the unpacked input."""
    N.require_cuda(x, w_ih, w_hh, b_ih, b_hh, what="WideGRU")
    _same_dtype("WideGRU", w_ih, x, w_hh, b_ih, b_hh)
    n = w_ih.shape[0]
    _packed_rnn_check(x, n, "WideGRU")
    hidden = w_hh.shape[2]
    if w_ih.shape[2] != x.shape[2] or tuple(w_hh.shape) != (n, 3 * hidden, hidden):
        raise ValueError(f"WideGRU: weights {tuple(w_ih.shape)} / {tuple(w_hh.shape)} do not match {tuple(x.shape)}")
    wi, wh = _dense(w_ih), _dense(w_hh)
    strides = (wi.shape[1] * wi.shape[2], wi.shape[2], wh.shape[1] * wh.shape[2], wh.shape[2])
    out, hn, _ = _rnn_fwd(False, x, None, None, wi, wh, _opt_dense(b_ih), _opt_dense(b_hh), strides, n, hidden,
                          packed=True)
    return out, hn


def lstm_blockdiag_packed(x: Tensor, weight_ih: Tensor, weight_hh: Tensor, b_ih: Optional[Tensor],
                          b_hh: Optional[Tensor], n: int, hidden: int):
    """WideLSTM forward (block-diagonal parameters, zero initial state) on the
    packed boundary layout: x [B, N*T, I] -> (out [B, N*T, H], (h_n, c_n))."""
    N.require_cuda(x, weight_ih, weight_hh, b_ih, b_hh, what="WideLSTM")
    _same_dtype("WideLSTM", weight_ih, x, weight_hh, b_ih, b_hh)
    _packed_rnn_check(x, n, "WideLSTM")
    inp = x.shape[2]
    if tuple(weight_ih.shape) != (n * 4 * hidden, n * inp) or tuple(weight_hh.shape) != (n * 4 * hidden, n * hidden):
        raise ValueError(f"WideLSTM: block-diagonal weights {tuple(weight_ih.shape)} / {tuple(weight_hh.shape)} do "
                         f"not match N={n}, I={inp}, H={hidden}")
    wi, wh = _dense(weight_ih), _dense(weight_hh)
    strides = (4 * hidden * n * inp + inp, n * inp, 4 * hidden * n * hidden + hidden, n * hidden)
    out, hn, cn = _rnn_fwd(True, x, None, None, wi, wh, _opt_dense(b_ih), _opt_dense(b_hh), strides, n, hidden,
                           packed=True)
    return out, (hn, cn)


def _opt_dense(t: Optional[Tensor]) -> Optional[Tensor]:
    return None if t is None else _dense(t)


def gru(x: Tensor, h0: Optional[Tensor], w_ih: Tensor, w_hh: Tensor, b_ih: Optional[Tensor],
        b_hh: Optional[Tensor]):
    """WideGRU forward: returns (out [N, B, T, H], h_n [N, B, H])."""
    if _compiling():
        return torch.ops.widek.gru(x, h0, w_ih, w_hh, b_ih, b_hh)
    if _AG.needs_grad(x, h0, w_ih, w_hh, b_ih, b_hh):
        return _AG.run(gru, _AG.gru_t, x, h0, w_ih, w_hh, b_ih, b_hh)
    N.require_cuda(x, h0, w_ih, w_hh, b_ih, b_hh, what="WideGRU")
    _same_dtype("WideGRU", w_ih, x, h0, w_hh, b_ih, b_hh)
    n, batch, steps, hidden = _rnn_check(x, w_ih, w_hh, 3, "WideGRU")
    if h0 is not None and tuple(h0.shape) != (n, batch, hidden):
        raise ValueError(f"WideGRU: h_0 must be [N, B, H] = {(n, batch, hidden)}, got {tuple(h0.shape)}")
    wi, wh = _dense(w_ih), _dense(w_hh)
    strides = (wi.shape[1] * wi.shape[2], wi.shape[2], wh.shape[1] * wh.shape[2], wh.shape[2])
    out, hn, _ = _rnn_fwd(False, x, _opt_dense(h0), None, wi, wh, _opt_dense(b_ih), _opt_dense(b_hh), strides, n,
                          hidden)
    return out, hn


def lstm_blockdiag(x: Tensor, h0: Optional[Tensor], c0: Optional[Tensor], weight_ih: Tensor, weight_hh: Tensor,
                   b_ih: Optional[Tensor], b_hh: Optional[Tensor], n: int, hidden: int):
    """WideLSTM forward straight from the block-diagonal module parameters
    weight_ih [n*4H, n*I] and weight_hh [n*4H, n*H] (model i's block read by
    stride, no extracted copy), biases [n, 4H]: (out, (h_n, c_n)). Returns
    None (launching nothing) when autograd needs the result."""
    if _compiling():
        out, hn, cn = torch.ops.widek.lstm(x, h0, c0, weight_ih, weight_hh, b_ih, b_hh, n, hidden)
        return out, (hn, cn)
    if _AG.needs_grad(x, h0, c0, weight_ih, weight_hh, b_ih, b_hh):
        return None
    N.require_cuda(x, h0, c0, weight_ih, weight_hh, b_ih, b_hh, what="WideLSTM")
    _same_dtype("WideLSTM", weight_ih, x, h0, c0, weight_hh, b_ih, b_hh)
    if x.dim() != 4 or x.shape[0] != n:
        raise ValueError(f"WideLSTM: input must be [N={n}, B, T, I], got {tuple(x.shape)}")
    inp, batch = x.shape[3], x.shape[1]
    if tuple(weight_ih.shape) != (n * 4 * hidden, n * inp) or tuple(weight_hh.shape) != (n * 4 * hidden, n * hidden):
        raise ValueError(f"WideLSTM: block-diagonal weights {tuple(weight_ih.shape)} / {tuple(weight_hh.shape)} do "
                         f"not match N={n}, I={inp}, H={hidden}")
    for name, t in (("h_0", h0), ("c_0", c0)):
        if t is not None and tuple(t.shape) != (n, batch, hidden):
            raise ValueError(f"WideLSTM: {name} must be [N, B, H] = {(n, batch, hidden)}, got {tuple(t.shape)}")
    wi, wh = _dense(weight_ih), _dense(weight_hh)
    strides = (4 * hidden * n * inp + inp, n * inp, 4 * hidden * n * hidden + hidden, n * hidden)
    out, hn, cn = _rnn_fwd(True, x, _opt_dense(h0), _opt_dense(c0), wi, wh, _opt_dense(b_ih), _opt_dense(b_hh),
                           strides, n, hidden)
    return out, (hn, cn)


def lstm(x: Tensor, h0: Optional[Tensor], c0: Optional[Tensor], w_ih: Tensor, w_hh: Tensor,
         b_ih: Optional[Tensor], b_hh: Optional[Tensor]):
    """WideLSTM forward on dense diagonal blocks w_ih [N, 4H, I],
    w_hh [N, 4H, H]: returns (out, (h_n, c_n))."""
    if _AG.needs_grad(x, h0, c0, w_ih, w_hh, b_ih, b_hh):
        out, hn, cn = _AG.run(_lstm_flat, _AG.lstm_t, x, h0, c0, w_ih, w_hh, b_ih, b_hh)
        return out, (hn, cn)
    N.require_cuda(x, h0, c0, w_ih, w_hh, b_ih, b_hh, what="WideLSTM")
    _same_dtype("WideLSTM", w_ih, x, h0, c0, w_hh, b_ih, b_hh)
    n, batch, steps, hidden = _rnn_check(x, w_ih, w_hh, 4, "WideLSTM")
    for name, t in (("h_0", h0), ("c_0", c0)):
        if t is not None and tuple(t.shape) != (n, batch, hidden):
            raise ValueError(f"WideLSTM: {name} must be [N, B, H] = {(n, batch, hidden)}, got {tuple(t.shape)}")
    wi, wh = _dense(w_ih), _dense(w_hh)
    strides = (wi.shape[1] * wi.shape[2], wi.shape[2], wh.shape[1] * wh.shape[2], wh.shape[2])
    out, hn, cn = _rnn_fwd(True, x, _opt_dense(h0), _opt_dense(c0), wi, wh, _opt_dense(b_ih), _opt_dense(b_hh),
                           strides, n, hidden)
    return out, (hn, cn)


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------

def _lstm_flat(x, h0, c0, w_ih, w_hh, b_ih, b_hh):
    out, (hn, cn) = lstm(x, h0, c0, w_ih, w_hh, b_ih, b_hh)
    return out, hn, cn


def attention_core(q: Tensor, k: Tensor, v: Tensor, nb: int, heads: int, tq: int, tk: int, head_dim: int,
                   q_stride: int, k_stride: int, v_stride: int, out: Tensor, causal: bool,
                   attn_mask: Optional[Tensor]) -> Tensor:
    """softmax(q k^T / sqrt(head_dim) [+mask]) v over nb*heads heads, reading
    q/k/v through row strides (elements; the tensors passed are the base
    views) and writing ``out`` rows of heads*head_dim elements."""
    dev = out.device
    kind, mptr, strides = 0, None, None
    keep_alive = None
    if attn_mask is not None:
        m = attn_mask.to(dev)
        if m.dtype == torch.bool:
            m = m.view(torch.uint8)
            kind = 1
        elif m.dtype == q.dtype:
            kind = 2
        else:
            m = m.to(torch.float32)
            kind = 3
        try:
            m4 = torch.broadcast_to(m, (nb, heads, tq, tk))
        except RuntimeError:
            raise ValueError(f"WideAttention: attn_mask of shape {tuple(attn_mask.shape)} does not broadcast to "
                             f"[N*B={nb}, heads={heads}, Tq={tq}, Tk={tk}]") from None
        keep_alive = m4
        mptr = m4.data_ptr()
        strides = (ctypes.c_int64 * 4)(*m4.stride())
    with _guard(dev):
        rc = N.lib().widek_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), q_stride,
                                         k_stride, v_stride, heads * head_dim, nb, heads, tq, tk, head_dim,
                                         1 if causal else 0, mptr, kind, strides, 1.0 / math.sqrt(head_dim),
                                         N.dtype_code(out), N.stream_ptr(dev))
    del keep_alive
    N.check(rc, "widek_attention_fwd")
    return out


def fused_qkv(q_weight: Tensor, kv_weight: Tensor, q_bias: Optional[Tensor],
              kv_bias: Optional[Tensor]):
    """[q; kv] weight [N, 3D, D] (and bias [N, 3D]) for self-attention, kept
    on q_weight between calls while the four parameters are unchanged
    (``_derived``: rebuilt after in-place updates and inside every CUDA-graph
    capture)."""
    def build():
        with torch.no_grad():
            w = torch.cat([q_weight, kv_weight], dim=1).contiguous()
            b = None if q_bias is None else torch.cat([q_bias, kv_bias], dim=1).contiguous()
        return w, b
    return _derived.cached(q_weight, 'qkv', (q_weight, kv_weight, q_bias, kv_bias), build)


def attention_tensors(query: Tensor, key: Tensor, value: Tensor, q_weight: Tensor, q_bias: Optional[Tensor],
                      kv_weight: Tensor, kv_bias: Optional[Tensor], out_weight: Tensor, out_bias: Optional[Tensor],
                      n_heads: int, attn_mask: Optional[Tensor], is_causal: bool, self_attn: bool,
                      out_ln=None) -> Tensor:
    """WideAttention forward on N-first [N, B, T, D] tensors from its
    parameters: q_weight [N, D, D], kv_weight [N, 2D, D] (k rows then v rows),
    out_weight [N, D, D], biases [N, D] / [N, 2D]; self_attn: key and value
    are the query (one fused [q; kv] projection)."""
    params = (q_weight, q_bias, kv_weight, kv_bias, out_weight, out_bias)
    if out_ln is not None and (_compiling() or _AG.needs_grad(query, key, value, *params, out_ln[0], out_ln[1])):
        # traced or differentiated: the two ops, each on its own operator
        y = attention_tensors(query, key, value, *params, n_heads, attn_mask, is_causal, self_attn)
        return layernorm(y, out_ln[0], out_ln[1], q_weight.shape[0], q_weight.shape[1], out_ln[2])
    if _compiling():
        return torch.ops.widek.attention(query, key, value, q_weight, q_bias, kv_weight, kv_bias, out_weight,
                                         out_bias, n_heads, attn_mask, is_causal, self_attn)
    if _AG.needs_grad(query, key, value, *params):
        kernel = lambda q, k, v, m, c, h, *p: attention_tensors(q, k, v, *p, h, m, c, self_attn)
        return _AG.run(kernel, _AG.attention_t, query, key, value, attn_mask, is_causal, n_heads, *params)
    dev = N.require_cuda(query, key, value, q_weight, what="WideAttention")
    _same_dtype("WideAttention", q_weight, query, key, value)
    if is_causal and attn_mask is not None:
        raise RuntimeError("WideAttention: an explicit attn_mask cannot be combined with is_causal=True "
                           "(same rule as scaled_dot_product_attention)")
    n, d = q_weight.shape[0], q_weight.shape[1]
    heads = n_heads
    dh = d // heads
    if query.dim() != 4 or query.shape[0] != n or query.shape[3] != d:
        raise ValueError(f"WideAttention: query must be [N={n}, B, T, D={d}], got {tuple(query.shape)}")
    _, b, tq, _ = query.shape
    tk = key.shape[2]
    if key.shape[:2] != (n, b) or value.shape[:3] != key.shape[:3]:
        raise ValueError("WideAttention: key/value shapes do not match the query")
    if self_attn:
        w, bias = fused_qkv(q_weight, kv_weight, q_bias, kv_bias)
        qkv = linear(query, w, bias)                       # [N, B, T, 3D]
        flat = qkv.view(-1)
        q_t, k_t, v_t = flat, flat[d:], flat[2 * d:]
        sq = sk = sv = 3 * d
    elif value is key:
        q_t = linear(query, q_weight, q_bias).view(-1)
        kv = linear(key, kv_weight, kv_bias).view(-1)      # [N, B, Tk, 2D]
        k_t, v_t = kv, kv[d:]
        sq, sk, sv = d, 2 * d, 2 * d
    else:
        kb = kv_bias
        q_t = linear(query, q_weight, q_bias).view(-1)
        k_t = linear(key, kv_weight[:, :d], None if kb is None else kb[:, :d]).view(-1)
        v_t = linear(value, kv_weight[:, d:], None if kb is None else kb[:, d:]).view(-1)
        sq = sk = sv = d
    o = torch.empty(n, b, tq, d, device=dev, dtype=query.dtype)
    attention_core(q_t, k_t, v_t, n * b, heads, tq, tk, dh, sq, sk, sv, o, is_causal, attn_mask)
    return _out_projection(o, out_weight, out_bias, out_ln, False)


def _out_projection(o: Tensor, out_weight: Tensor, out_bias: Optional[Tensor], out_ln, out_packed: bool) -> Tensor:
    """The attention output projection; with ``out_ln`` = (weight, bias, eps)
    of a WideLayerNorm that follows it, the LayerNorm too (one launch where
    the fused kernel takes the shapes, else the two ops)."""
    if out_ln is not None:
        y = linear_ln_layout(o, out_weight, out_bias, out_ln[0], out_ln[1], out_ln[2], False, out_packed)
        if y is not None:
            return y
        n, d = out_weight.shape[0], out_weight.shape[1]
        if out_packed:
            y = linear_layout(o, out_weight, out_bias, ACT_NONE, False, True)
            return layernorm_packed(y, out_ln[0], out_ln[1], n, d, out_ln[2])
        return layernorm(linear(o, out_weight, out_bias), out_ln[0], out_ln[1], n, d, out_ln[2])
    if out_packed:
        return linear_layout(o, out_weight, out_bias, ACT_NONE, False, True)
    return linear(o, out_weight, out_bias)


def attention_packed(mod, x: Tensor, is_causal: bool, out_ln=None) -> Tensor:
    """WideAttention self-attention on the packed boundary layout: x
    [B, N*T, D] -> [B, N*T, D], the fused QKV projection reading the packed
    rows in place and the output projection writing them packed; equal to
    unpacking, ``attention_tensors`` and packing (traced_wide.py:463-469,
    :527-532 around wide_attention.py:178-238)."""
    n, d = mod.q_weight.shape[0], mod.q_weight.shape[1]
    heads = mod.n_heads
    if x.dim() != 3 or x.shape[1] % n != 0 or x.shape[2] != d:
        raise ValueError(f"WideAttention: packed input must be [B, N*T, D={d}] with N={n}, got {tuple(x.shape)}")
    dev = N.require_cuda(x, mod.q_weight, what="WideAttention")
    b, t = x.shape[0], x.shape[1] // n
    w, bias = fused_qkv(mod.q_weight, mod.kv_weight, mod.q_bias, mod.kv_bias)
    qkv = linear_layout(x, w, bias, ACT_NONE, True, False)      # [N, B, T, 3D]
    flat = qkv.view(-1)
    o = torch.empty(n, b, t, d, device=dev, dtype=x.dtype)
    attention_core(flat, flat[d:], flat[2 * d:], n * b, heads, t, t, d // heads, 3 * d, 3 * d, 3 * d, o, is_causal,
                   None)
    return _out_projection(o, mod.out_weight, mod.out_bias, out_ln, True)


def attention(mod, query: Tensor, key: Tensor, value: Tensor, attn_mask: Optional[Tensor], is_causal: bool,
              out_ln=None) -> Tensor:
    """WideAttention forward on N-first [N, B, T, D] tensors (see the module);
    ``out_ln`` = (weight, bias, eps) of a WideLayerNorm applied to the result
    fuses it into the output projection."""
    return attention_tensors(query, key, value, mod.q_weight, mod.q_bias, mod.kv_weight, mod.kv_bias,
                             mod.out_weight, mod.out_bias, mod.n_heads, attn_mask, is_causal,
                             key is query and value is query, out_ln)


def attention_dropout(mod, query: Tensor, key: Tensor, value: Tensor, attn_mask: Optional[Tensor],
                      is_causal: bool, dropout_p: float) -> Tensor:
    """WideAttention in training mode with attention dropout
    (wide_attention.py:221-228 of the reference, which passes
    ``dropout_p = self.dropout`` to scaled_dot_product_attention while
    training). The Q, K, V and output projections run on the WideLinear
    kernels (with their backward kernels under autograd); the core with its
    random mask runs on torch's ``scaled_dot_product_attention`` on the GPU,
    whose backward reuses the mask its forward drew from torch's generator,
    so a seeded run draws the same mask as the reference's. Rows with no
    attended key follow SDPA here (NaN), not the kernels' zeros."""
    import torch.nn.functional as F
    N.require_cuda(query, key, value, mod.q_weight, what="WideAttention")
    _same_dtype("WideAttention", mod.q_weight, query, key, value)
    if is_causal and attn_mask is not None:
        raise RuntimeError("WideAttention: an explicit attn_mask cannot be combined with is_causal=True "
                           "(same rule as scaled_dot_product_attention)")
    n, d, heads = mod.n, mod.d_model, mod.n_heads
    dh = d // heads
    if query.dim() != 4 or query.shape[0] != n or query.shape[3] != d:
        raise ValueError(f"WideAttention: query must be [N={n}, B, T, D={d}], got {tuple(query.shape)}")
    _, b, tq, _ = query.shape
    tk = key.shape[2]
    if key.shape[:2] != (n, b) or value.shape[:3] != key.shape[:3]:
        raise ValueError("WideAttention: key/value shapes do not match the query")
    kv_b = mod.kv_bias
    q = linear(query, mod.q_weight, mod.q_bias)
    k = linear(key, mod.kv_weight[:, :d], None if kv_b is None else kv_b[:, :d])
    v = linear(value, mod.kv_weight[:, d:], None if kv_b is None else kv_b[:, d:])
    heads_of = lambda t, tt: t.reshape(n * b, tt, heads, dh).transpose(1, 2)
    mask = None if attn_mask is None else attn_mask.to(query.device)    # as the kernel path (attention_core)
    o = F.scaled_dot_product_attention(heads_of(q, tq), heads_of(k, tk), heads_of(v, tk), attn_mask=mask,
                                       dropout_p=dropout_p, is_causal=is_causal, scale=1.0 / math.sqrt(dh))
    return linear(o.transpose(1, 2).reshape(n, b, tq, d), mod.out_weight, mod.out_bias)


# ---------------------------------------------------------------------------
# Convolutions
# ---------------------------------------------------------------------------

def _packed_weight(weight: Tensor, rows: int, cin: int, taps: int, dev) -> Tensor:
    """[rows, cin, taps] -> [rows, taps, cin_p] (cin_p = cin rounded up to 64,
    zero-filled) for the tensor-core conv, kept on the weight tensor between
    forwards (see ``_derived``: rebuilt when its version, storage, dtype or
    shape changes, and inside every CUDA-graph capture)."""
    def build():
        wd = _dense(weight.detach())
        elems = int(N.lib().widek_conv_packed_weight_elems(rows, cin, taps))
        wp = torch.empty(elems, device=dev, dtype=weight.dtype)
        with _guard(dev):
            rc = N.lib().widek_conv_pack_weight(wd.data_ptr(), wp.data_ptr(), rows, cin, taps, wd.element_size(),
                                                N.stream_ptr(dev))
        N.check(rc, "widek_conv_pack_weight")
        return wp
    return _derived.cached(weight, 'conv_packed', (weight,), build, extra=(rows, cin, taps))


LAYOUT_NFIRST, LAYOUT_PACKED, LAYOUT_CLAST = 0, 1, 2
CONV_PATH_DIRECT, CONV_PATH_TAPS, CONV_PATH_HALO = 0, 1, 2


def conv_geometry(n, batch, cin, cout, sp_in, kernel, stride, padding, dilation):
    """The 22-entry geometry array of the conv entry points (spatial values
    padded to 3-D) and the padded input spatial, kernel, stride and the
    output spatial of the given rank."""
    nd = len(sp_in)
    pad3 = lambda v, fill: (fill,) * (3 - nd) + tuple(v)
    sp = pad3(sp_in, 1)
    ks = pad3(kernel, 1)
    st = pad3(stride, 1)
    pd = pad3(padding, 0)
    dl = pad3(dilation, 1)
    out_sp = tuple((sp[i] + 2 * pd[i] - dl[i] * (ks[i] - 1) - 1) // st[i] + 1 for i in range(3))
    if min(out_sp) <= 0:
        raise ValueError(f"WideConv: output size {out_sp} is not positive")
    geom = (ctypes.c_int64 * 22)(n, batch, cin, cout, *sp, *ks, *st, *pd, *dl, *out_sp)
    return geom, sp, ks, st, out_sp[3 - nd:]


_TC_PATH_CACHE: dict = {}


def _tensor_core_path(geom, dtype_code: int, in_layout: int, out_layout: int, res_layout: int,
                      has_residual: bool) -> bool:
    """Whether the library runs this conv on a tensor-core kernel (which then
    needs the packed weights and, for a non-channels-last input, the staging
    workspace). The library's own decision (widek_conv_path), memoised."""
    key = (tuple(geom), dtype_code, in_layout, out_layout, res_layout, has_residual)
    hit = _TC_PATH_CACHE.get(key)
    if hit is None:
        path = int(N.lib().widek_conv_path(geom, dtype_code, in_layout, out_layout, res_layout,
                                           1 if has_residual else 0))
        hit = path in (CONV_PATH_TAPS, CONV_PATH_HALO)
        if len(_TC_PATH_CACHE) > 4096:
            _TC_PATH_CACHE.clear()
        _TC_PATH_CACHE[key] = hit
    return hit


def conv_path(n, batch, cin, cout, sp_in, kernel, stride, padding, dilation, dtype: torch.dtype,
              in_layout: int = LAYOUT_NFIRST, out_layout: int = LAYOUT_NFIRST, res_layout: int = LAYOUT_NFIRST,
              has_residual: bool = False) -> int:
    """Which kernel the library would run for this conv (CONV_PATH_*), or -1
    when the layout combination is not served. Launches nothing."""
    geom = conv_geometry(n, batch, cin, cout, sp_in, kernel, stride, padding, dilation)[0]
    code = N._DTYPE_CODES.get(dtype)
    if code is None:
        return -1
    return int(N.lib().widek_conv_path(geom, code, in_layout, out_layout, res_layout, 1 if has_residual else 0))


def conv_nd(x: Tensor, weight: Tensor, bias: Optional[Tensor], n: int, stride, padding, dilation,
            scale: Optional[Tensor] = None, shift: Optional[Tensor] = None, residual: Optional[Tensor] = None,
            act: int = ACT_NONE, residual_first: bool = False, in_layout: int = LAYOUT_NFIRST,
            out_layout: int = LAYOUT_NFIRST, res_layout: int = LAYOUT_NFIRST) -> Optional[Tensor]:
    """N independent convolutions with weight [N*Cout, Cin, *K] (1-3 spatial
    dims). x is [N, B, Cin, *S] (LAYOUT_NFIRST), [B, N*Cin, *S] (LAYOUT_PACKED,
    the TracedWideModel boundary layout) or [N, B, *S, Cin] (LAYOUT_CLAST); the
    result uses out_layout likewise, and the optional residual res_layout
    (NFIRST or PACKED). Optional fused epilogue: per-channel scale/shift
    ([N*Cout]), activation, residual. With non-default layouts the call
    returns None when the library cannot serve the combination for this
    geometry (nothing is launched); the default layouts always run."""
    if _compiling() and scale is None and shift is None and residual is None and act == ACT_NONE \
            and in_layout == out_layout == res_layout == LAYOUT_NFIRST:
        return torch.ops.widek.conv(x, weight, bias, n, list(stride), list(padding), list(dilation))
    if _AG.needs_grad(x, weight, bias, scale, shift, residual):
        return _AG.run(conv_nd, _AG.conv_nd_t, x, weight, bias, n, stride, padding, dilation, scale, shift,
                       residual, act, residual_first, in_layout, out_layout, res_layout)
    dev = N.require_cuda(x, weight, bias, scale, shift, residual, what="WideConv")
    _same_dtype("WideConv", weight, x, bias, scale, shift, residual)
    if in_layout == LAYOUT_PACKED:
        batch, cin, sp_in = x.shape[0], x.shape[1] // n, tuple(x.shape[2:])
        if x.shape[1] % n != 0:
            raise ValueError(f"WideConv: packed input {tuple(x.shape)} is not N={n} channel groups")
    elif in_layout == LAYOUT_CLAST:
        nn_, batch, cin, sp_in = x.shape[0], x.shape[1], x.shape[-1], tuple(x.shape[2:-1])
        if nn_ != n:
            raise ValueError(f"WideConv: channels-last input {tuple(x.shape)} is not N={n} models")
    else:
        nn_, batch, cin, sp_in = x.shape[0], x.shape[1], x.shape[2], tuple(x.shape[3:])
        if nn_ != n:
            raise ValueError(f"WideConv: input {tuple(x.shape)} does not match weight {tuple(weight.shape)} for N={n}")
    nd = len(sp_in)
    if nd not in (1, 2, 3) or weight.dim() != nd + 2:
        raise ValueError(f"WideConv: input {tuple(x.shape)} / weight {tuple(weight.shape)} rank mismatch")
    if weight.shape[0] % n != 0 or weight.shape[1] != cin:
        raise ValueError(f"WideConv: input {tuple(x.shape)} does not match weight {tuple(weight.shape)} for N={n}")
    cout = weight.shape[0] // n
    geom, sp, ks, st, osp = conv_geometry(n, batch, cin, cout, sp_in, weight.shape[2:], stride, padding, dilation)
    default = in_layout == out_layout == res_layout == LAYOUT_NFIRST
    if not default and not N.lib().widek_conv_layouts_supported(geom, N.dtype_code(x), in_layout, out_layout,
                                                                  res_layout, 1 if residual is not None else 0):
        return None
    if out_layout == LAYOUT_PACKED:
        y = torch.empty((batch, n * cout, *osp), device=dev, dtype=x.dtype)
    elif out_layout == LAYOUT_CLAST:
        y = torch.empty((n, batch, *osp, cout), device=dev, dtype=x.dtype)
    else:
        y = torch.empty((n, batch, cout, *osp), device=dev, dtype=x.dtype)
    xd = _dense(x)
    wp = ws = None
    if _tensor_core_path(geom, N.dtype_code(x), in_layout, out_layout, res_layout, residual is not None):
        taps = ks[0] * ks[1] * ks[2]
        wp = _packed_weight(weight, n * cout, cin, taps, dev)
        if in_layout != LAYOUT_CLAST:
            ws = torch.empty(int(N.lib().widek_conv_workspace(n, batch, cin, *sp, N.dtype_code(x))) //
                             x.element_size(), device=dev, dtype=x.dtype)
    with _guard(dev):
        rc = N.lib().widek_conv_fwd_ex(xd.data_ptr(), _dense(weight).data_ptr(), N.ptr(wp), N.ptr(bias),
                                       N.ptr(scale), N.ptr(shift),
                                       N.ptr(_dense(residual) if residual is not None else None),
                                       y.data_ptr(), N.ptr(ws), 0 if ws is None else ws.numel() * ws.element_size(),
                                       geom, act, 1 if residual_first else 0, in_layout, out_layout, res_layout,
                                       N.dtype_code(x), N.stream_ptr(dev))
    N.check(rc, "widek_conv_fwd")
    return y
