"""Generates the golden fixtures under tests/golden/ by running the REFERENCE
implementation (WideCompiler v0.6.0, imported from its source tree as
``ref_wide_compiler``) on seeded CPU inputs in fp32.

Each fixture ``<case>.pt`` is a dict:
    kind      which primitive / graph
    meta      constructor arguments and flags
    state     the reference wide module's state_dict (this repository's
              primitives use the same parameter layout, so it loads as is)
    inputs    input tensors
    outputs   reference outputs (and updated running stats where relevant)

Usage:  python tests/golden/make_golden.py [--root /path/to/reference] [--only forward|grads|traced_seq]
The fixtures are small (a few hundred KB in total) and committed.
"""
from __future__ import annotations

import argparse
import zlib
import os
import sys

import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import refimport  # noqa: E402


def _save(name, kind, meta, state, inputs, outputs):
    torch.save({'kind': kind, 'meta': meta, 'state': {k: v.clone() for k, v in state.items()},
                'inputs': inputs, 'outputs': outputs}, os.path.join(HERE, f"{name}.pt"))
    print(f"  {name}.pt")


def make_all(root: str) -> None:
    ref = refimport.load(root)
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False

    # --- WideLinear (wide_linear.py) -------------------------------------
    for name, (n, shape, i, o, bias) in {
        'linear_basic': (5, (7,), 24, 40, True),
        'linear_nobias_3d': (3, (2, 5), 16, 9, False),
        'linear_n1': (1, (4,), 8, 8, True),
    }.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        mods = [nn.Linear(i, o, bias=bias) for _ in range(n)]
        w = ref.WideLinear.from_modules(mods, strategy='einsum')
        x = torch.randn(n, *shape, i)
        _save(name, 'linear', {'n': n, 'in': i, 'out': o, 'bias': bias}, w.state_dict(), {'x': x},
              {'y': w(x).detach()})

    # --- WideLayerNorm (wide_layernorm.py) --------------------------------
    torch.manual_seed(11)
    n, d = 4, 48
    mods = [nn.LayerNorm(d) for _ in range(n)]
    for m in mods:
        with torch.no_grad():
            m.weight.uniform_(0.5, 1.5)
            m.bias.normal_(0, 0.1)
    w = ref.WideLayerNorm.from_modules(mods)
    x = torch.randn(n, 3, 5, d) * 2 + 0.5
    _save('layernorm', 'layernorm', {'n': n, 'd': d, 'eps': 1e-5}, w.state_dict(), {'x': x}, {'y': w(x).detach()})

    # --- BatchNorm2d / 1d (wide_batchnorm_2d.py / _1d.py) -----------------
    def bn_mods(cls, n, c):
        mods = [cls(c) for _ in range(n)]
        for m in mods:
            with torch.no_grad():
                m.running_mean.normal_(0, 1)
                m.running_var.uniform_(0.5, 2.0)
                m.weight.uniform_(0.5, 1.5)
                m.bias.normal_(0, 0.1)
        return mods

    for name, (cls, wcls, shape, train) in {
        'bn2d_eval': (nn.BatchNorm2d, ref.WideBatchNorm2d, (3, 4, 6, 5, 7), False),
        'bn2d_train': (nn.BatchNorm2d, ref.WideBatchNorm2d, (3, 4, 6, 5, 7), True),
        'bn1d_eval_3d': (nn.BatchNorm1d, ref.WideBatchNorm1d, (3, 8, 6), False),
        'bn1d_train_4d': (nn.BatchNorm1d, ref.WideBatchNorm1d, (2, 4, 5, 9), True),
    }.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        n, c = shape[0], shape[2]
        w = wcls.from_modules(bn_mods(cls, n, c))
        w.train(train)
        state0 = {k: v.clone() for k, v in w.state_dict().items()}
        x = torch.randn(*shape) * 1.5 + 0.3
        y = w(x).detach()
        _save(name, 'batchnorm', {'n': n, 'c': c, 'train': train, 'dims': len(shape)}, state0, {'x': x},
              {'y': y, 'running_mean': w.op.running_mean.clone(), 'running_var': w.op.running_var.clone(),
               'num_batches_tracked': w.op.num_batches_tracked.clone()})

    # --- GroupNorm (wide_groupnorm.py) -----------------------------------
    for name, (n, b, g, c, sp, affine) in {
        'groupnorm': (3, 2, 4, 8, (5, 6), True),
        'groupnorm_noaffine_1d': (2, 3, 2, 6, (7,), False),
    }.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        mods = [nn.GroupNorm(g, c, affine=affine) for _ in range(n)]
        if affine:
            for m in mods:
                with torch.no_grad():
                    m.weight.uniform_(0.5, 1.5)
                    m.bias.normal_(0, 0.1)
        w = ref.WideGroupNorm.from_modules(mods)
        x = torch.randn(n, b, c, *sp)
        _save(name, 'groupnorm', {'n': n, 'groups': g, 'c': c, 'affine': affine}, w.state_dict(), {'x': x},
              {'y': w(x).detach()})

    # --- InstanceNorm1d/2d (wide_instancenorm.py) -------------------------
    for name, (cls, wcls, shape, affine) in {
        'instnorm2d': (nn.InstanceNorm2d, ref.WideInstanceNorm2d, (3, 2, 4, 5, 6), False),
        'instnorm1d_affine': (nn.InstanceNorm1d, ref.WideInstanceNorm1d, (2, 3, 5, 11), True),
    }.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        n, c = shape[0], shape[2]
        mods = [cls(c, affine=affine) for _ in range(n)]
        if affine:
            for m in mods:
                with torch.no_grad():
                    m.weight.uniform_(0.5, 1.5)
                    m.bias.normal_(0, 0.1)
        w = wcls.from_modules(mods)
        x = torch.randn(*shape)
        _save(name, 'instancenorm', {'n': n, 'c': c, 'affine': affine, 'dims': len(shape)}, w.state_dict(),
              {'x': x}, {'y': w(x).detach()})

    # --- Embedding (wide_embedding.py) -----------------------------------
    torch.manual_seed(5)
    mods = [nn.Embedding(11, 6) for _ in range(3)]
    w = ref.WideEmbedding.from_modules(mods)
    idx = torch.randint(0, 11, (2, 5))
    _save('embedding', 'embedding', {'n': 3, 'v': 11, 'd': 6}, w.state_dict(), {'idx': idx},
          {'y': w(idx).detach()})

    # --- Convolutions (wide_conv1d/2d/3d.py) ------------------------------
    for name, (dims, n, b, cin, cout, k, s, p, dl, sp, bias) in {
        'conv2d_3x3': (2, 3, 2, 4, 5, 3, 1, 1, 1, (8, 8), True),
        'conv2d_stride2_dil2': (2, 2, 2, 3, 6, 3, 2, 2, 2, (9, 10), False),
        'conv2d_1x1': (2, 4, 3, 8, 4, 1, 1, 0, 1, (5, 5), True),
        'conv1d_k5': (1, 3, 2, 4, 6, 5, 1, 2, 1, (17,), True),
        'conv3d_3x3x3': (3, 2, 2, 3, 4, 3, 1, 1, 1, (4, 5, 6), True),
    }.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        cls = {1: nn.Conv1d, 2: nn.Conv2d, 3: nn.Conv3d}[dims]
        wcls = {1: ref.WideConv1d, 2: ref.WideConv2d, 3: ref.WideConv3d}[dims]
        mods = [cls(cin, cout, k, stride=s, padding=p, dilation=dl, bias=bias) for _ in range(n)]
        if dims == 2:
            w = wcls.from_modules(mods, strategy='grouped')
        elif dims == 1:
            w = wcls.from_modules(mods, strategy=ref.core.primitives.wide_conv1d.Conv1dStrategy.GROUPED)
        else:
            w = wcls.from_modules(mods, strategy='grouped')
        x = torch.randn(n, b, cin, *sp)
        _save(name, 'conv', {'dims': dims, 'n': n, 'cin': cin, 'cout': cout, 'k': k, 's': s, 'p': p, 'd': dl,
                             'bias': bias}, w.state_dict(), {'x': x}, {'y': w(x).detach()})

    # --- Attention (wide_attention.py) -----------------------------------
    for name, (n, b, tq, tk, d, h, causal, cross, mask) in {
        'attn_self': (2, 2, 9, 9, 16, 4, False, False, None),
        'attn_causal': (3, 2, 12, 12, 32, 2, True, False, None),
        'attn_cross': (2, 3, 7, 5, 16, 2, False, True, None),
        'attn_mask_float': (2, 2, 6, 6, 16, 4, False, False, 'float'),
        'attn_mask_bool': (2, 2, 6, 6, 16, 4, False, False, 'bool'),
    }.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        mods = [nn.MultiheadAttention(d, h, batch_first=True) for _ in range(n)]
        for m in mods:
            with torch.no_grad():
                m.in_proj_bias.normal_(0, 0.1)
                m.out_proj.bias.normal_(0, 0.1)
        w = ref.WideAttention.from_modules(mods).eval()
        q = torch.randn(n, b, tq, d)
        k = torch.randn(n, b, tk, d) if cross else None
        v = torch.randn(n, b, tk, d) if cross else None
        am = None
        if mask == 'float':
            am = torch.randn(tq, tk)
        elif mask == 'bool':
            am = torch.rand(tq, tk) > 0.3
            am[:, 0] = True
        with torch.no_grad():
            out = w(q, k, v, attn_mask=am, is_causal=causal)
        y = out[0] if isinstance(out, tuple) else out
        _save(name, 'attention', {'n': n, 'd': d, 'heads': h, 'causal': causal, 'cross': cross,
                                  'tuple': isinstance(out, tuple)}, w.state_dict(),
              {'q': q, 'k': k, 'v': v, 'mask': am}, {'y': y.detach()})

    # --- GRU / LSTM (wide_gru.py / wide_lstm.py) --------------------------
    for name, (cell, n, b, t, i, hs, with_h0) in {
        'gru': ('gru', 3, 2, 5, 6, 8, False),
        'gru_h0': ('gru', 2, 3, 4, 5, 12, True),
        'lstm': ('lstm', 3, 2, 5, 6, 8, False),
        'lstm_h0': ('lstm', 2, 3, 4, 5, 12, True),
    }.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        if cell == 'gru':
            mods = [nn.GRU(i, hs, batch_first=True) for _ in range(n)]
            w = ref.WideGRU.from_modules(mods)
            x = torch.randn(n, b, t, i)
            h0 = torch.randn(n, b, hs) if with_h0 else None
            with torch.no_grad():
                out, hn = w(x, h0)
            _save(name, 'gru', {'n': n, 'i': i, 'h': hs}, w.state_dict(), {'x': x, 'h0': h0},
                  {'y': out, 'h_n': hn})
        else:
            mods = [nn.LSTM(i, hs, batch_first=True) for _ in range(n)]
            w = ref.WideLSTM.from_modules(mods)
            x = torch.randn(n, b, t, i)
            hx = (torch.randn(n, b, hs), torch.randn(n, b, hs)) if with_h0 else None
            with torch.no_grad():
                out, (hn, cn) = w(x, hx)
            _save(name, 'lstm', {'n': n, 'i': i, 'h': hs}, w.state_dict(),
                  {'x': x, 'h0': hx[0] if hx else None, 'c0': hx[1] if hx else None},
                  {'y': out, 'h_n': hn, 'c_n': cn})

    # --- TracedWideModel graphs (traced_wide.py) --------------------------
    class MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1 = nn.Linear(8, 16)
            self.fc2 = nn.Linear(16, 8)

        def forward(self, x):
            return self.fc2(F.relu(self.fc1(x)))

    class ResBlock(nn.Module):
        def __init__(self, c=4):
            super().__init__()
            self.conv1 = nn.Conv2d(c, c, 3, padding=1)
            self.bn1 = nn.BatchNorm2d(c)
            self.conv2 = nn.Conv2d(c, c, 3, padding=1)
            self.bn2 = nn.BatchNorm2d(c)

        def forward(self, x):
            h = F.relu(self.bn1(self.conv1(x)))
            return self.bn2(self.conv2(h)) + x

    for name, (cls, n, shape) in {'traced_mlp': (MLP, 4, (3, 8)), 'traced_resblock': (ResBlock, 2, (2, 4, 6, 6))}.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        models = [cls().eval() for _ in range(n)]
        for m in models:
            for mod in m.modules():
                if isinstance(mod, nn.BatchNorm2d):
                    with torch.no_grad():
                        mod.running_mean.normal_(0, 1)
                        mod.running_var.uniform_(0.5, 2.0)
                        mod.weight.uniform_(0.5, 1.5)
                        mod.bias.normal_(0, 0.1)
        wide = ref.TracedWideModel.from_models(models, torch.randn(*shape)).eval()
        inputs = [torch.randn(*shape) for _ in range(n)]
        packed = ref.pack_inputs(inputs)
        with torch.no_grad():
            out = wide(packed)
        _save(name, 'traced', {'n': n, 'model': cls.__name__},
              {f"m{k}.{key}": v for k, m in enumerate(models) for key, v in m.state_dict().items()},
              {'inputs': inputs, 'packed': packed}, {'y': out})


def make_grads(root: str) -> None:
    """Gradient fixtures: the reference's modules differentiated by torch
    autograd (the reference's training path; its gradient-flow test is
    wide_lstm.py:744-762) with a seeded upstream gradient dy, i.e.
    d(sum(y * dy)) with respect to the input and every parameter."""
    ref = refimport.load(root)
    torch.backends.cuda.matmul.allow_tf32 = False

    # WideLinear (wide_linear.py:162-171), then an optional activation the
    # way a traced graph applies it (torch.relu / F.gelu on the wide output)
    for name, (n, shape, i, o, bias, act) in {
        'grad_linear_basic': (4, (9,), 24, 40, True, 'none'),
        'grad_linear_gelu_3d': (3, (2, 5), 16, 12, True, 'gelu'),
        'grad_linear_relu_nobias': (2, (7,), 20, 8, False, 'relu'),
    }.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        mods = [nn.Linear(i, o, bias=bias) for _ in range(n)]
        w = ref.WideLinear.from_modules(mods, strategy='einsum')
        x = torch.randn(n, *shape, i, requires_grad=True)
        y = w(x)
        y = {'none': lambda t: t, 'relu': torch.relu, 'gelu': F.gelu}[act](y)
        dy = torch.randn_like(y)
        (y * dy).sum().backward()
        grads = {'x': x.grad.clone()}
        for k, v in w.named_parameters():
            grads[k] = v.grad.clone()
        _save(name, 'grad_linear', {'n': n, 'in': i, 'out': o, 'bias': bias, 'act': act}, w.state_dict(),
              {'x': x.detach(), 'dy': dy}, {'y': y.detach(), 'grads': grads})

    # WideLayerNorm (wide_layernorm.py:62-65)
    torch.manual_seed(21)
    n, d = 3, 40
    mods = [nn.LayerNorm(d) for _ in range(n)]
    for m in mods:
        with torch.no_grad():
            m.weight.uniform_(0.5, 1.5)
            m.bias.normal_(0, 0.1)
    w = ref.WideLayerNorm.from_modules(mods)
    x = (torch.randn(n, 4, 6, d) * 2 + 0.5).requires_grad_(True)
    y = w(x)
    dy = torch.randn_like(y)
    (y * dy).sum().backward()
    grads = {'x': x.grad.clone()}
    for k, v in w.named_parameters():
        grads[k] = v.grad.clone()
    _save('grad_layernorm', 'grad_layernorm', {'n': n, 'd': d, 'eps': 1e-5}, w.state_dict(),
          {'x': x.detach(), 'dy': dy}, {'y': y.detach(), 'grads': grads})

    # WideBatchNorm2d (wide_batchnorm_2d.py:53-72), training (batch
    # statistics) and eval (running statistics)
    for name, train in {'grad_bn2d_train': True, 'grad_bn2d_eval': False}.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        n, c = 3, 4
        mods = [nn.BatchNorm2d(c) for _ in range(n)]
        for m in mods:
            with torch.no_grad():
                m.running_mean.normal_(0, 1)
                m.running_var.uniform_(0.5, 2.0)
                m.weight.uniform_(0.5, 1.5)
                m.bias.normal_(0, 0.1)
        w = ref.WideBatchNorm2d.from_modules(mods)
        w.train(train)
        state0 = {k: v.clone() for k, v in w.state_dict().items()}
        x = (torch.randn(n, 5, c, 6, 7) * 1.5 + 0.3).requires_grad_(True)
        y = w(x)
        dy = torch.randn_like(y)
        (y * dy).sum().backward()
        grads = {'x': x.grad.clone()}
        for k, v in w.named_parameters():
            grads[k] = v.grad.clone()
        _save(name, 'grad_batchnorm', {'n': n, 'c': c, 'train': train, 'eps': 1e-5}, state0,
              {'x': x.detach(), 'dy': dy}, {'y': y.detach(), 'grads': grads})

    # WideGroupNorm (wide_groupnorm.py:90-117)
    torch.manual_seed(31)
    n, b, g, c = 3, 2, 4, 8
    mods = [nn.GroupNorm(g, c) for _ in range(n)]
    for m in mods:
        with torch.no_grad():
            m.weight.uniform_(0.5, 1.5)
            m.bias.normal_(0, 0.1)
    w = ref.WideGroupNorm.from_modules(mods)
    x = (torch.randn(n, b, c, 5, 6) * 2 + 0.5).requires_grad_(True)
    y = w(x)
    dy = torch.randn_like(y)
    (y * dy).sum().backward()
    grads = {'x': x.grad.clone()}
    for k, v in w.named_parameters():
        grads[k] = v.grad.clone()
    _save('grad_groupnorm', 'grad_groupnorm', {'n': n, 'groups': g, 'c': c, 'eps': 1e-5}, w.state_dict(),
          {'x': x.detach(), 'dy': dy}, {'y': y.detach(), 'grads': grads})


class AttnLN(nn.Module):
    """cfg5's model, small: causal self-attention, then LayerNorm."""

    def __init__(self, d=16, heads=2):
        super().__init__()
        self.attn = nn.MultiheadAttention(d, heads, batch_first=True)
        self.ln = nn.LayerNorm(d)

    def forward(self, x):
        a, _ = self.attn(x, x, x, need_weights=False, is_causal=True)
        return self.ln(a)


class GRUOut(nn.Module):
    def __init__(self, i=6, h=10):
        super().__init__()
        self.gru = nn.GRU(i, h, batch_first=True)

    def forward(self, x):
        out, _ = self.gru(x)
        return out


class LSTMOut(nn.Module):
    def __init__(self, i=6, h=10):
        super().__init__()
        self.lstm = nn.LSTM(i, h, batch_first=True)

    def forward(self, x):
        out, _ = self.lstm(x)
        return out


SEQ_GRAPHS = {'traced_attn_ln': (AttnLN, 3, (2, 12, 16), {'heads': 2, 'causal': True}),
              'traced_gru': (GRUOut, 3, (2, 5, 6), {}), 'traced_lstm': (LSTMOut, 2, (3, 4, 6), {})}


def make_traced_seq(root: str) -> None:
    """TracedWideModel graphs of the sequence primitives (reference
    traced_wide.py:450-534 around wide_attention.py / wide_gru.py /
    wide_lstm.py): attention -> getitem -> LayerNorm (cfg5's graph, causal)
    and a recurrent layer -> getitem, on packed inputs [B, N*T, F]."""
    ref = refimport.load(root)
    torch.backends.cuda.matmul.allow_tf32 = False
    for name, (cls, n, shape, extra) in SEQ_GRAPHS.items():
        torch.manual_seed(zlib.crc32(name.encode()) % 1000)
        models = [cls().eval() for _ in range(n)]
        for m in models:
            for mod in m.modules():
                if isinstance(mod, nn.LayerNorm):
                    with torch.no_grad():
                        mod.weight.uniform_(0.5, 1.5)
                        mod.bias.normal_(0, 0.1)
                if isinstance(mod, nn.MultiheadAttention):
                    with torch.no_grad():
                        mod.in_proj_bias.normal_(0, 0.1)
                        mod.out_proj.bias.normal_(0, 0.1)
        wide = ref.TracedWideModel.from_models(models, torch.randn(*shape)).eval()
        inputs = [torch.randn(*shape) for _ in range(n)]
        packed = ref.pack_inputs(inputs)
        with torch.no_grad():
            out = wide(packed)
        _save(name, 'traced', {'n': n, 'model': cls.__name__, **extra},
              {f"m{k}.{key}": v for k, m in enumerate(models) for key, v in m.state_dict().items()},
              {'inputs': inputs, 'packed': packed}, {'y': out})


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--root', default=refimport.DEFAULT_ROOT)
    ap.add_argument('--only', choices=['forward', 'grads', 'traced_seq'], default=None,
                    help="generate only the forward, the gradient or the traced sequence-model fixtures")
    a = ap.parse_args()
    if not refimport.available(a.root):
        sys.exit(f"reference not found under {a.root!r}: pass --root or set WIDE_REFERENCE_ROOT to the "
                 "checkout that holds wide_compiler/")
    if a.only in (None, 'forward'):
        make_all(a.root)
    if a.only in (None, 'grads'):
        make_grads(a.root)
    if a.only in (None, 'traced_seq'):
        make_traced_seq(a.root)
