"""CPU oracle for the wide-primitive forward path — TEST INFRASTRUCTURE ONLY.

This module restates, in explicit float64 torch-CPU arithmetic, what each
reference primitive computes (WideCompiler v0.6.0, a pure-Python/PyTorch
package; the arithmetic lives in its torch calls). It is the checker for the
CUDA kernels: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg may import it. The product (``wide_compiler``) never does.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference itself
(imported from its source tree) on seeded inputs and stores inputs,
parameters and outputs under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks every function here against those fixtures.

All functions take N-first tensors and the primitive's parameters as plain
tensors, compute in float64 and return float64 results (callers cast).
Citations are path:line inside the reference project.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor

D = torch.float64


def _f(t: Optional[Tensor]) -> Optional[Tensor]:
    return None if t is None else t.detach().to('cpu', D)


# ---------------------------------------------------------------------------
# Linear — wide_compiler/core/primitives/wide_linear.py:150-173
#   out[n] = x[n] @ weight[n]^T + bias[n]   (einsum 'noi,nbi->nbo' + bias)
# ---------------------------------------------------------------------------
def linear(x: Tensor, weight: Tensor, bias: Optional[Tensor], act: str = 'none') -> Tensor:
    x, w, b = _f(x), _f(weight), _f(bias)
    n, o, k = w.shape
    batch = x.shape[1:-1]
    y = torch.bmm(x.reshape(n, -1, k), w.transpose(1, 2))
    if b is not None:
        y = y + b[:, None, :]
    y = activation(y, act)
    return y.reshape(n, *batch, o)


def activation(x: Tensor, act: str) -> Tensor:
    """Elementwise glue of traced_wide.py:174-186 (FunctionalOp) in float64."""
    if act == 'none':
        return x
    if act == 'relu':
        return torch.clamp_min(x, 0.0)
    if act == 'gelu':
        return 0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0)))
    if act == 'sigmoid':
        return 1.0 / (1.0 + torch.exp(-x))
    if act == 'tanh':
        return torch.tanh(x)
    if act == 'silu':
        return x / (1.0 + torch.exp(-x))
    raise ValueError(act)


def binary(a: Tensor, b: Tensor, op: str) -> Tensor:
    """BinaryOp (traced_wide.py:189-211)."""
    a, b = _f(a), _f(b)
    return {'add': a + b, 'mul': a * b, 'sub': a - b, 'div': a / b}[op]


# ---------------------------------------------------------------------------
# LayerNorm — wide_layernorm.py:41-67
#   mean over last dim, biased variance, (x-mean)/sqrt(var+eps)*w[n]+b[n]
# ---------------------------------------------------------------------------
def layernorm(x: Tensor, weight_flat: Tensor, bias_flat: Tensor, n: int, d: int, eps: float) -> Tensor:
    x = _f(x)
    w = _f(weight_flat).view(n, *([1] * (x.dim() - 2)), d)
    b = _f(bias_flat).view(n, *([1] * (x.dim() - 2)), d)
    mean = x.mean(dim=-1, keepdim=True)
    var = ((x - mean) ** 2).mean(dim=-1, keepdim=True)
    return (x - mean) / torch.sqrt(var + eps) * w + b


# ---------------------------------------------------------------------------
# Gradients (the reference trains by torch autograd over the forwards above;
# its gradient-flow test: wide_lstm.py:744-762). Explicit formulas in
# float64, the upstream gradient dy given:
#   WideLinear + act:  dpre = dy * act'(pre)  (ReLU: 1 where the output is
#                      > 0; GELU: Phi(pre) + pre * phi(pre)),
#                      dx = dpre W, dW = sum_rows dpre^T x, db = sum_rows dpre
#   WideLayerNorm:     g = dy * gamma,
#                      dx = rstd * (g - mean(g) - x_hat * mean(g * x_hat)),
#                      dgamma = sum_rows dy * x_hat, dbeta = sum_rows dy
# ---------------------------------------------------------------------------
def linear_grads(x: Tensor, weight: Tensor, bias: Optional[Tensor], dy: Tensor, act: str = 'none'):
    """(dx, dweight, dbias or None) of activation(linear(x, weight, bias))."""
    x, w, b, g = _f(x), _f(weight), _f(bias), _f(dy)
    n, o, k = w.shape
    x2 = x.reshape(n, -1, k)
    pre = torch.bmm(x2, w.transpose(1, 2))
    if b is not None:
        pre = pre + b[:, None, :]
    g2 = g.reshape(n, -1, o)
    if act == 'relu':
        g2 = g2 * (pre > 0).to(D)
    elif act == 'gelu':
        g2 = g2 * (0.5 * (1.0 + torch.erf(pre / math.sqrt(2.0))) + pre * torch.exp(-0.5 * pre * pre)
                   / math.sqrt(2.0 * math.pi))
    elif act != 'none':
        raise ValueError(act)
    dx = torch.bmm(g2, w).reshape(x.shape)
    dw = torch.bmm(g2.transpose(1, 2), x2)
    db = g2.sum(dim=1) if b is not None else None
    return dx, dw, db


def layernorm_grads(x: Tensor, weight_flat: Tensor, dy: Tensor, n: int, d: int, eps: float):
    """(dx, dweight_flat, dbias_flat) of layernorm(x, weight_flat, ., n, d, eps)."""
    x, g = _f(x), _f(dy)
    w = _f(weight_flat).view(n, *([1] * (x.dim() - 2)), d)
    mean = x.mean(dim=-1, keepdim=True)
    var = ((x - mean) ** 2).mean(dim=-1, keepdim=True)
    rstd = 1.0 / torch.sqrt(var + eps)
    xh = (x - mean) * rstd
    gg = g * w
    dx = rstd * (gg - gg.mean(dim=-1, keepdim=True) - xh * (gg * xh).mean(dim=-1, keepdim=True))
    rows = tuple(range(1, x.dim() - 1))
    dw = (g * xh).sum(dim=rows).reshape(n * d) if rows else (g * xh).reshape(n * d)
    db = g.sum(dim=rows).reshape(n * d) if rows else g.reshape(n * d)
    return dx, dw, db


def _norm_grads(x: Tensor, g: Tensor, gamma: Tensor, dims, mean: Tensor, rstd: Tensor, batch_stats: bool):
    """dx, and the per-element dy * x_hat, for a normalisation whose
    statistics reduce over `dims`: with batch statistics
    dx = rstd * (g' - mean(g') - x_hat * mean(g' * x_hat)), g' = dy * gamma;
    with fixed (running) statistics dx = rstd * g'."""
    xh = (x - mean) * rstd
    gg = g * gamma
    if batch_stats:
        dx = rstd * (gg - gg.mean(dim=dims, keepdim=True) - xh * (gg * xh).mean(dim=dims, keepdim=True))
    else:
        dx = rstd * gg
    return dx, g * xh


def batchnorm_grads(x: Tensor, n: int, c: int, weight: Optional[Tensor], running_mean: Optional[Tensor],
                    running_var: Optional[Tensor], dy: Tensor, batch_stats: bool, eps: float):
    """(dx, dweight_flat or None, dbias_flat) of batchnorm on [N, B, C, *S]
    (batch statistics: biased variance over B and S per (model, channel))."""
    x, g = _f(x), _f(dy)
    shape = (n, 1, c) + (1,) * (x.dim() - 3)
    dims = tuple([1] + list(range(3, x.dim())))
    if batch_stats:
        mean = x.mean(dim=dims, keepdim=True)
        var = ((x - mean) ** 2).mean(dim=dims, keepdim=True)
    else:
        mean, var = _f(running_mean).view(shape), _f(running_var).view(shape)
    rstd = 1.0 / torch.sqrt(var + eps)
    gamma = _f(weight).view(shape) if weight is not None else torch.ones(shape, dtype=D)
    dx, gxh = _norm_grads(x, g, gamma, dims, mean, rstd, batch_stats)
    dw = gxh.sum(dim=dims).reshape(n * c) if weight is not None else None
    return dx, dw, g.sum(dim=dims).reshape(n * c)


def groupnorm_grads(x: Tensor, n: int, groups: int, weight: Optional[Tensor], dy: Tensor, eps: float):
    """(dx, dweight_flat or None, dbias_flat) of groupnorm on [N, B, C, *S]
    (statistics per (model, sample, group))."""
    x, g = _f(x), _f(dy)
    b, c = x.shape[1], x.shape[2]
    xg = x.reshape(n, b, groups, -1)
    mean = xg.mean(dim=-1, keepdim=True)
    var = ((xg - mean) ** 2).mean(dim=-1, keepdim=True)
    rstd = 1.0 / torch.sqrt(var + eps)
    cshape = (n, 1, c) + (1,) * (x.dim() - 3)
    gamma = (_f(weight).view(cshape) if weight is not None else torch.ones(cshape, dtype=D)).expand(x.shape)
    dxg, gxh = _norm_grads(xg, g.reshape(n, b, groups, -1), gamma.reshape(n, b, groups, -1), (-1,), mean, rstd,
                           True)
    rows = tuple([1] + list(range(3, x.dim())))
    dw = gxh.reshape(x.shape).sum(dim=rows).reshape(n * c) if weight is not None else None
    return dxg.reshape(x.shape), dw, g.sum(dim=rows).reshape(n * c)


# ---------------------------------------------------------------------------
# BatchNorm1d/2d — wide_batchnorm_2d.py:53-72, wide_batchnorm_1d.py:53-73
# (inner nn.BatchNorm over N*C channels == per-(model, channel) statistics)
# ---------------------------------------------------------------------------
def batchnorm(x: Tensor, n: int, c: int, weight: Optional[Tensor], bias: Optional[Tensor],
              running_mean: Optional[Tensor], running_var: Optional[Tensor], use_batch_stats: bool,
              momentum: float = 0.1, eps: float = 1e-5) -> Tuple[Tensor, Optional[Tensor], Optional[Tensor]]:
    """Returns (y, new_running_mean, new_running_var); running stats are
    updated only when use_batch_stats and they are given (torch semantics:
    rm = (1-m)*rm + m*mean, rv = (1-m)*rv + m*var_unbiased)."""
    x = _f(x)
    shp = x.shape                                    # [N, B, C, *S]
    xr = x.reshape(n, shp[1], c, -1)                 # [N, B, C, L]
    if use_batch_stats:
        mean = xr.mean(dim=(1, 3))                   # [N, C]
        var = ((xr - mean[:, None, :, None]) ** 2).mean(dim=(1, 3))
        cnt = xr.shape[1] * xr.shape[3]
    else:
        mean = _f(running_mean).view(n, c)
        var = _f(running_var).view(n, c)
    y = (xr - mean[:, None, :, None]) / torch.sqrt(var[:, None, :, None] + eps)
    if weight is not None:
        y = y * _f(weight).view(n, 1, c, 1)
    if bias is not None:
        y = y + _f(bias).view(n, 1, c, 1)
    new_rm = new_rv = None
    if use_batch_stats and running_mean is not None:
        unbiased = var * cnt / max(cnt - 1, 1)
        new_rm = (1 - momentum) * _f(running_mean) + momentum * mean.reshape(-1)
        new_rv = (1 - momentum) * _f(running_var) + momentum * unbiased.reshape(-1)
    return y.reshape(shp), new_rm, new_rv


# ---------------------------------------------------------------------------
# GroupNorm — wide_groupnorm.py:90-117 (nn.GroupNorm(N*G, N*C) on the
# channel-packed tensor == statistics per (model, sample, group))
# InstanceNorm — wide_instancenorm.py:89-108, :222-240 (G == C)
# ---------------------------------------------------------------------------
def groupnorm(x: Tensor, n: int, groups: int, weight: Optional[Tensor], bias: Optional[Tensor],
              eps: float) -> Tensor:
    x = _f(x)
    shp = x.shape
    c = shp[2]
    xr = x.reshape(n, shp[1], groups, -1)
    mean = xr.mean(dim=-1, keepdim=True)
    var = ((xr - mean) ** 2).mean(dim=-1, keepdim=True)
    y = ((xr - mean) / torch.sqrt(var + eps)).reshape(n, shp[1], c, -1)
    if weight is not None:
        y = y * _f(weight).view(n, 1, c, 1)
    if bias is not None:
        y = y + _f(bias).view(n, 1, c, 1)
    return y.reshape(shp)


# ---------------------------------------------------------------------------
# Embedding — wide_embedding.py:85-99 (weight[:, idx] -> [N, *idx.shape, D])
# ---------------------------------------------------------------------------
def embedding(idx: Tensor, weight: Tensor) -> Tensor:
    return _f(weight)[:, idx.to('cpu', torch.long)]


# ---------------------------------------------------------------------------
# Convolution — wide_conv2d.py:169-194 (grouped conv, groups=N, on the
# channel-packed tensor == one conv per model); wide_conv1d.py, wide_conv3d.py
# ---------------------------------------------------------------------------
def conv_nd(x: Tensor, weight: Tensor, bias: Optional[Tensor], n: int, stride: Sequence[int],
            padding: Sequence[int], dilation: Sequence[int]) -> Tensor:
    x, w, b = _f(x), _f(weight), _f(bias)
    nd = x.dim() - 3
    conv = {1: F.conv1d, 2: F.conv2d, 3: F.conv3d}[nd]
    cout = w.shape[0] // n
    outs = []
    for i in range(n):
        bi = None if b is None else b[i * cout:(i + 1) * cout]
        outs.append(conv(x[i], w[i * cout:(i + 1) * cout], bi, stride=tuple(stride), padding=tuple(padding),
                         dilation=tuple(dilation)))
    return torch.stack(outs)


# ---------------------------------------------------------------------------
# Attention — wide_attention.py:178-238
#   q = x_q Wq^T + bq, k = x_k Wk^T + bk, v = x_v Wv^T + bv (Wk = kv[:D],
#   Wv = kv[D:]); per head softmax(q k^T / sqrt(dh) [+mask | causal]) v;
#   merge heads; out = o Wo^T + bo.
# ---------------------------------------------------------------------------
def attention(query: Tensor, key: Tensor, value: Tensor, q_weight: Tensor, kv_weight: Tensor,
              q_bias: Optional[Tensor], kv_bias: Optional[Tensor], out_weight: Tensor, out_bias: Optional[Tensor],
              n_heads: int, attn_mask: Optional[Tensor] = None, is_causal: bool = False) -> Tensor:
    qx, kx, vx = _f(query), _f(key), _f(value)
    wq, wkv, wo = _f(q_weight), _f(kv_weight), _f(out_weight)
    n, b, tq, d = qx.shape
    tk = kx.shape[2]
    dh = d // n_heads
    q = torch.einsum('nbtd,nod->nbto', qx, wq)
    k = torch.einsum('nbtd,nod->nbto', kx, wkv[:, :d])
    v = torch.einsum('nbtd,nod->nbto', vx, wkv[:, d:])
    if q_bias is not None:
        q = q + _f(q_bias)[:, None, None, :]
        k = k + _f(kv_bias)[:, None, None, :d]
        v = v + _f(kv_bias)[:, None, None, d:]
    q = q.view(n, b, tq, n_heads, dh).transpose(2, 3)
    k = k.view(n, b, tk, n_heads, dh).transpose(2, 3)
    v = v.view(n, b, tk, n_heads, dh).transpose(2, 3)
    s = q @ k.transpose(-1, -2) / math.sqrt(dh)
    if is_causal:
        keep = torch.ones(tq, tk, dtype=torch.bool).tril()
        s = s.masked_fill(~keep, float('-inf'))
    if attn_mask is not None:
        # SDPA broadcasts the mask against [N*B, heads, tq, tk].
        m = torch.broadcast_to(attn_mask.to('cpu'), (n * b, n_heads, tq, tk)).reshape(n, b, n_heads, tq, tk)
        if m.dtype == torch.bool:
            s = s.masked_fill(~m, float('-inf'))
        else:
            s = s + m.to(D)
    p = torch.softmax(s, dim=-1)
    o = (p @ v).transpose(2, 3).reshape(n, b, tq, d)
    out = torch.einsum('nbtd,nod->nbto', o, wo)
    if out_bias is not None:
        out = out + _f(out_bias)[:, None, None, :]
    return out


# ---------------------------------------------------------------------------
# GRU — wide_gru.py:148-213 (gate order r, z, n)
# ---------------------------------------------------------------------------
def gru(x: Tensor, h0: Optional[Tensor], w_ih: Tensor, w_hh: Tensor, b_ih: Optional[Tensor],
        b_hh: Optional[Tensor]) -> Tuple[Tensor, Tensor]:
    x, w_ih, w_hh, b_ih, b_hh = _f(x), _f(w_ih), _f(w_hh), _f(b_ih), _f(b_hh)
    n, b, t, _ = x.shape
    hsz = w_hh.shape[2]
    gx = torch.einsum('nbti,ngi->nbtg', x, w_ih)
    if b_ih is not None:
        gx = gx + b_ih[:, None, None, :]
    h = torch.zeros(n, b, hsz, dtype=D) if h0 is None else _f(h0)
    outs = []
    for step in range(t):
        gh = torch.einsum('nbh,ngh->nbg', h, w_hh)
        if b_hh is not None:
            gh = gh + b_hh[:, None, :]
        xr, xz, xn = gx[:, :, step].chunk(3, dim=-1)
        hr, hz, hn = gh.chunk(3, dim=-1)
        r = torch.sigmoid(xr + hr)
        z = torch.sigmoid(xz + hz)
        nn_ = torch.tanh(xn + r * hn)
        h = (1 - z) * nn_ + z * h
        outs.append(h)
    return torch.stack(outs, dim=2), h


# ---------------------------------------------------------------------------
# LSTM — wide_lstm.py:158-234 (gate order i, f, g, o; dense diagonal blocks)
# ---------------------------------------------------------------------------
def lstm(x: Tensor, h0: Optional[Tensor], c0: Optional[Tensor], w_ih: Tensor, w_hh: Tensor,
         b_ih: Optional[Tensor], b_hh: Optional[Tensor]) -> Tuple[Tensor, Tuple[Tensor, Tensor]]:
    """w_ih [N, 4H, I], w_hh [N, 4H, H] (the block-diagonal layout's blocks),
    b_ih/b_hh [N, 4H]."""
    x, w_ih, w_hh, b_ih, b_hh = _f(x), _f(w_ih), _f(w_hh), _f(b_ih), _f(b_hh)
    n, b, t, _ = x.shape
    hsz = w_hh.shape[2]
    gx = torch.einsum('nbti,ngi->nbtg', x, w_ih)
    if b_ih is not None:
        gx = gx + b_ih[:, None, None, :]
    h = torch.zeros(n, b, hsz, dtype=D) if h0 is None else _f(h0)
    c = torch.zeros(n, b, hsz, dtype=D) if c0 is None else _f(c0)
    outs = []
    for step in range(t):
        g = gx[:, :, step] + torch.einsum('nbh,ngh->nbg', h, w_hh)
        if b_hh is not None:
            g = g + b_hh[:, None, :]
        i_, f_, g_, o_ = g.chunk(4, dim=-1)
        c = torch.sigmoid(f_) * c + torch.sigmoid(i_) * torch.tanh(g_)
        h = torch.sigmoid(o_) * torch.tanh(c)
        outs.append(h)
    return torch.stack(outs, dim=2), (h, c)


def lstm_blocks(weight_ih: Tensor, weight_hh: Tensor, n: int) -> Tuple[Tensor, Tensor]:
    """Diagonal blocks of the block-diagonal LSTM weights (wide_lstm.py:184-199)."""
    four_h = weight_ih.shape[0] // n
    i = weight_ih.shape[1] // n
    h = weight_hh.shape[1] // n
    bih = torch.stack([weight_ih[k * four_h:(k + 1) * four_h, k * i:(k + 1) * i] for k in range(n)])
    bhh = torch.stack([weight_hh[k * four_h:(k + 1) * four_h, k * h:(k + 1) * h] for k in range(n)])
    return bih, bhh


# ---------------------------------------------------------------------------
# Layout boundary — ensemble_util.py:20-101, traced_wide.py:463-469, :527-532
# ---------------------------------------------------------------------------
def pack_inputs(inputs: Sequence[Tensor]) -> Tensor:
    st = torch.stack([t.detach().cpu() for t in inputs], dim=1)
    b, n = st.shape[0], st.shape[1]
    rest = st.shape[2:]
    return st.reshape(b, n) if not rest else st.reshape(b, n * rest[0], *rest[1:])


def packed_to_nfirst(x: Tensor, n: int) -> Tensor:
    b, nc = x.shape[0], x.shape[1]
    return x.detach().cpu().reshape(b, n, nc // n, *x.shape[2:]).movedim(1, 0).contiguous()


def nfirst_to_packed(x: Tensor) -> Tensor:
    n, b, c = x.shape[0], x.shape[1], x.shape[2]
    return x.detach().cpu().movedim(0, 1).reshape(b, n * c, *x.shape[3:])


# ---------------------------------------------------------------------------
# The benchmark model graphs, composed from the functions above
# ---------------------------------------------------------------------------
def mlp2(x_packed: Tensor, n: int, w1: Tensor, b1: Tensor, w2: Tensor, b2: Tensor) -> Tensor:
    """TracedWideModel of N two-layer MLPs (Linear -> ReLU -> Linear),
    channel-packed in and out (traced_wide.py:450-534)."""
    x = packed_to_nfirst(x_packed, n)
    h = linear(x, w1, b1, act='relu')
    return nfirst_to_packed(linear(h, w2, b2))


def resblock(x: Tensor, n: int, c1w: Tensor, c1b: Optional[Tensor], bn1: dict, c2w: Tensor,
             c2b: Optional[Tensor], bn2: dict) -> Tensor:
    """N-first ResBlock: conv3x3 -> BN(eval) -> ReLU -> conv3x3 -> BN(eval) + x."""
    h = conv_nd(x, c1w, c1b, n, (1, 1), (1, 1), (1, 1))
    c = h.shape[2]
    h, _, _ = batchnorm(h, n, c, bn1['weight'], bn1['bias'], bn1['running_mean'], bn1['running_var'], False,
                        eps=bn1.get('eps', 1e-5))
    h = torch.clamp_min(h, 0.0)
    h = conv_nd(h, c2w, c2b, n, (1, 1), (1, 1), (1, 1))
    h, _, _ = batchnorm(h, n, c, bn2['weight'], bn2['bias'], bn2['running_mean'], bn2['running_var'], False,
                        eps=bn2.get('eps', 1e-5))
    return h + _f(x)


def linear_ref_dtype(x: Tensor, weight: Tensor, bias: Optional[Tensor]) -> Tensor:
    """The reference's own op sequence for WideLinear (wide_linear.py:162-171:
    einsum 'noi,nbi->nbo', then + bias[:, None]) in the INPUT dtype, on the
    host. Used only to time the reference's CPU path (bench.py cpu_baseline
    and --impl reference), not as a parity checker."""
    n, o, k = weight.shape
    out = torch.einsum('noi,nbi->nbo', weight, x.reshape(n, -1, k))
    if bias is not None:
        out = out + bias.unsqueeze(1)
    return out


# ---------------------------------------------------------------------------
# The reference's own op sequences in the storage dtype, for timing the
# reference's CPU path in bench.py (not parity checkers).
# ---------------------------------------------------------------------------
def mlp2_ref_dtype(x_nfirst: Tensor, w1, b1, w2, b2) -> Tensor:
    """TracedWideModel MLP stages: WideLinear (einsum + bias), F.relu, WideLinear."""
    return linear_ref_dtype(torch.relu(linear_ref_dtype(x_nfirst, w1, b1)), w2, b2)


def resblock_ref_dtype(x: Tensor, c1w, c1b, bn1, c2w, c2b, bn2) -> Tensor:
    """WideConv2d (permute + grouped conv, wide_conv2d.py:169-194),
    WideBatchNorm2d eval (wide_batchnorm_2d.py:53-72), ReLU, conv, BN, + x."""
    n, b, c, h, w = x.shape

    def conv(t, wt, bs):
        p = t.permute(1, 0, 2, 3, 4).reshape(b, n * c, h, w)
        o = F.conv2d(p, wt, bs, padding=1, groups=n)
        return o.view(b, n, c, h, w).permute(1, 0, 2, 3, 4).contiguous()

    def bn(t, prm):
        p = t.permute(1, 0, 2, 3, 4).reshape(b, n * c, h, w)
        o = F.batch_norm(p, prm['running_mean'], prm['running_var'], prm['weight'], prm['bias'], False, 0.0, 1e-5)
        return o.view(b, n, c, h, w).permute(1, 0, 2, 3, 4).contiguous()

    hdn = torch.relu(bn(conv(x, c1w, c1b), bn1))
    return bn(conv(hdn, c2w, c2b), bn2) + x


def gru_ref_dtype(x, w_ih, w_hh, b_ih, b_hh):
    """wide_gru.py:148-213 op sequence in the input dtype."""
    n, b, t, _ = x.shape
    hsz = w_hh.shape[2]
    gx = torch.einsum('nbti,ngi->nbtg', x, w_ih) + b_ih.view(n, 1, 1, -1)
    h = torch.zeros(n, b, hsz, dtype=x.dtype)
    outs = []
    for s in range(t):
        gh = torch.einsum('nbh,ngh->nbg', h, w_hh) + b_hh.view(n, 1, -1)
        xr, xz, xn = gx[:, :, s].chunk(3, dim=-1)
        hr, hz, hn = gh.chunk(3, dim=-1)
        r = torch.sigmoid(xr + hr)
        z = torch.sigmoid(xz + hz)
        h = (1 - z) * torch.tanh(xn + r * hn) + z * h
        outs.append(h)
    return torch.stack(outs, dim=2), h


def lstm_ref_dtype(x, w_ih, w_hh, b_ih, b_hh):
    """wide_lstm.py:158-234 op sequence (diagonal blocks) in the input dtype."""
    n, b, t, _ = x.shape
    hsz = w_hh.shape[2]
    gx = torch.einsum('nbti,ngi->nbtg', x, w_ih) + b_ih.view(n, 1, 1, -1)
    h = torch.zeros(n, b, hsz, dtype=x.dtype)
    c = torch.zeros(n, b, hsz, dtype=x.dtype)
    outs = []
    for s in range(t):
        g = gx[:, :, s] + torch.einsum('nbh,ngh->nbg', h, w_hh) + b_hh.view(n, 1, -1)
        i_, f_, g_, o_ = g.chunk(4, dim=-1)
        c = torch.sigmoid(f_) * c + torch.sigmoid(i_) * torch.tanh(g_)
        h = torch.sigmoid(o_) * torch.tanh(c)
        outs.append(h)
    return torch.stack(outs, dim=2), (h, c)


def attention_ln_ref_dtype(x, q_weight, kv_weight, out_weight, heads, ln_w, ln_b, eps=1e-5):
    """wide_attention.py:178-238 (einsum projections, head split,
    F.scaled_dot_product_attention causal, merge, out projection) followed by
    wide_layernorm.py:41-67, in the input dtype (biases are zero in cfg5)."""
    n, b, t, d = x.shape
    dh = d // heads
    q = torch.einsum('nbtd,nod->nbto', x, q_weight)
    k = torch.einsum('nbtd,nod->nbto', x, kv_weight[:, :d])
    v = torch.einsum('nbtd,nod->nbto', x, kv_weight[:, d:])
    sp = lambda u: u.view(n, b, t, heads, dh).permute(0, 1, 3, 2, 4).reshape(n * b, heads, t, dh)
    o = F.scaled_dot_product_attention(sp(q), sp(k), sp(v), is_causal=True)
    o = o.view(n, b, heads, t, dh).permute(0, 1, 3, 2, 4).reshape(n, b, t, d)
    y = torch.einsum('nbtd,nod->nbto', o, out_weight)
    mean = y.mean(dim=-1, keepdim=True)
    var = y.var(dim=-1, unbiased=False, keepdim=True)
    return (y - mean) / torch.sqrt(var + eps) * ln_w.view(n, 1, 1, d) + ln_b.view(n, 1, 1, d)


def batchnorm2d_ref_dtype(x, running_mean, running_var, weight, bias, training, momentum=0.1, eps=1e-5):
    """wide_batchnorm_2d.py:53-72 in the input dtype: permute to the
    channel-packed [B, N*C, H, W] layout, nn.BatchNorm2d(N*C) (batch
    statistics and the running update when training), permute back."""
    n, b, c, h, w = x.shape
    p = x.permute(1, 0, 2, 3, 4).reshape(b, n * c, h, w)
    o = F.batch_norm(p, running_mean, running_var, weight, bias, training, momentum, eps)
    return o.view(b, n, c, h, w).permute(1, 0, 2, 3, 4).contiguous()


def groupnorm_ref_dtype(x, groups, weight, bias, eps=1e-5):
    """wide_groupnorm.py:90-117 in the input dtype: channel-packed
    nn.GroupNorm(N*G, N*C), then back to N-first."""
    n, b, c = x.shape[:3]
    sp = x.shape[3:]
    p = x.permute(1, 0, 2, *range(3, x.dim())).reshape(b, n * c, *sp)
    o = F.group_norm(p, n * groups, weight, bias, eps)
    return o.view(b, n, c, *sp).permute(1, 0, 2, *range(3, x.dim())).contiguous()


def layernorm_ref_dtype(x, weight_flat, bias_flat, n, d, eps=1e-5):
    """wide_layernorm.py:41-67 in the input dtype (mean, biased var, divide
    by sqrt, per-model affine)."""
    wgt = weight_flat.view(n, *([1] * (x.dim() - 2)), d)
    bs = bias_flat.view(n, *([1] * (x.dim() - 2)), d)
    mean = x.mean(dim=-1, keepdim=True)
    var = x.var(dim=-1, unbiased=False, keepdim=True)
    return (x - mean) / torch.sqrt(var + eps) * wgt + bs
