"""GPU parity after parameter updates: a model compiled with compile=True
(the CUDA-graph executor) must follow every change of its parameters made
after a graph was recorded, as torch.compile's wrapper in the reference
does (wide_compiler/api.py:137-147): in-place arithmetic (``mul_``),
``load_state_dict`` (in-place copies), and writes through ``.data``. The
kernels read derived copies of some parameters (repacked conv weights, the
folded eval BatchNorm, the fused [q; kv] attention projection, the LSTM
diagonal blocks); each case below changes a parameter behind one of them and
checks the next replay against the oracle computed from the live
parameters, and against the eager model."""
import pytest
import torch
import torch.nn as nn

import wide_compiler as wc
from gpu_util import assert_fp32_close, assert_lowp_close, no_device_error
from oracle import wide_oracle as O

pytestmark = pytest.mark.gpu
DEV = 'cuda'
BF = torch.bfloat16


# ---------------------------------------------------------------------------
# conv + BatchNorm (the cfg3 block, small)
# ---------------------------------------------------------------------------

class _Block(nn.Module):
    def __init__(self, c=64):
        super().__init__()
        self.conv1 = nn.Conv2d(c, c, 3, padding=1)
        self.bn1 = nn.BatchNorm2d(c)
        self.conv2 = nn.Conv2d(c, c, 3, padding=1)
        self.bn2 = nn.BatchNorm2d(c)

    def forward(self, x):
        return self.bn2(self.conv2(torch.relu(self.bn1(self.conv1(x))))) + x


def _bn_dict(bn):
    return {k: getattr(bn, k).detach().cpu() for k in ('weight', 'bias', 'running_mean', 'running_var')} | \
        {'eps': bn.eps}


def _block_oracle(wide, x, n):
    st = wide.stages
    xn = O.packed_to_nfirst(x, n)
    y = O.resblock(xn, n, st['conv1'].grouped_conv.weight.detach().cpu(), st['conv1'].grouped_conv.bias.detach().cpu(),
                   _bn_dict(st['bn1'].op), st['conv2'].grouped_conv.weight.detach().cpu(),
                   st['conv2'].grouped_conv.bias.detach().cpu(), _bn_dict(st['bn2'].op))
    return O.nfirst_to_packed(y)


def _block_models(n, c, seed):
    torch.manual_seed(seed)
    models = []
    for _ in range(n):
        m = _Block(c)
        with torch.no_grad():
            for bn in (m.bn1, m.bn2):
                bn.running_mean.normal_(0, 0.5)
                bn.running_var.uniform_(0.5, 2.0)
                bn.weight.uniform_(0.5, 1.5)
                bn.bias.normal_(0, 0.1)
        models.append(m.eval())
    return models


def test_graphed_conv_block_follows_parameter_updates():
    n, c, hw, b = 3, 64, 16, 2
    models = _block_models(n, c, 11)
    sample = torch.randn(1, c, hw, hw)
    graphed = wc.compile(models, sample, compile_model=True).to(DEV, BF).eval()
    eager = wc.compile(models, sample).to(DEV, BF).eval()
    x = torch.randn(b, n * c, hw, hw, device=DEV).to(BF)

    def check():
        y = graphed(x)
        assert len(graphed._graphs) == 1, "the update must not need a new recording"
        assert_lowp_close(y, _block_oracle(graphed._orig_mod, x, n))
        eager.load_state_dict(graphed._orig_mod.state_dict())
        assert_lowp_close(y, eager(x).double())

    with torch.no_grad():
        check()                                                   # records, replays
        check()                                                   # replays
        st = graphed._orig_mod.stages
        st['conv1'].grouped_conv.weight.mul_(0.5)                 # repacked conv weight
        check()
        st['bn1'].op.running_mean.add_(0.75)                      # folded BatchNorm
        st['bn2'].op.weight.mul_(-1.0)
        check()
        new = {k: (v * 1.25 if v.is_floating_point() and 'running_var' not in k else v)
               for k, v in graphed._orig_mod.state_dict().items()}
        graphed._orig_mod.load_state_dict(new)                    # in-place copies
        check()
        st['conv2'].grouped_conv.weight.data.copy_(torch.randn_like(st['conv2'].grouped_conv.weight) * 0.02)
        st['bn2'].op.running_var.data.mul_(3.0)                   # .data writes: no version bump
        y = graphed(x)
        assert_lowp_close(y, _block_oracle(graphed._orig_mod, x, n))
    no_device_error()


def test_eager_conv_block_after_data_writes_needs_invalidate():
    """Eager forwards key their caches on tensor versions; ``.data`` writes
    do not bump them, and ``invalidate_caches()`` makes the next forward
    rebuild every derived tensor."""
    n, c, hw, b = 2, 64, 16, 2
    models = _block_models(n, c, 12)
    wide = wc.compile(models, torch.randn(1, c, hw, hw)).to(DEV, BF).eval()
    x = torch.randn(b, n * c, hw, hw, device=DEV).to(BF)
    with torch.no_grad():
        y0 = wide(x).clone()
        assert_lowp_close(y0, _block_oracle(wide, x, n))
        bn = wide.stages['bn1'].op
        bn.weight.data.mul_(2.0)
        wide.stages['conv2'].grouped_conv.weight.data.mul_(-1.0)
        wide.invalidate_caches()
        y1 = wide(x)
        assert (y1.double() - y0.double()).abs().max() > 0.1
        assert_lowp_close(y1, _block_oracle(wide, x, n))
        bn.weight.mul_(0.25)                                       # version bump: no call needed
        assert_lowp_close(wide(x), _block_oracle(wide, x, n))
    no_device_error()


# ---------------------------------------------------------------------------
# attention -> LayerNorm (the cfg5 graph, small)
# ---------------------------------------------------------------------------

class _AttnLN(nn.Module):
    def __init__(self, d=128, heads=2):
        super().__init__()
        self.attn = nn.MultiheadAttention(d, heads, batch_first=True)
        self.ln = nn.LayerNorm(d)

    def forward(self, x):
        return self.ln(self.attn(x, x, x, need_weights=False)[0])


def _attn_oracle(wide, x, n):
    a, ln = wide.stages['attn'], wide.stages['ln']
    xn = O.packed_to_nfirst(x, n)
    g = lambda t: None if t is None else t.detach().cpu()
    y = O.attention(xn, xn, xn, g(a.q_weight), g(a.kv_weight), g(a.q_bias), g(a.kv_bias), g(a.out_weight),
                    g(a.out_bias), a.n_heads)
    y = O.layernorm(y, g(ln.weight), g(ln.bias), n, a.d_model, ln.eps)
    return O.nfirst_to_packed(y)


def test_graphed_attention_follows_parameter_updates():
    n, d, t, b = 3, 128, 128, 2
    torch.manual_seed(13)
    models = [_AttnLN(d).eval() for _ in range(n)]
    for m in models:
        with torch.no_grad():
            m.attn.in_proj_bias.normal_(0, 0.1)
            m.ln.weight.uniform_(0.5, 1.5)
    sample = torch.randn(1, t, d)
    graphed = wc.compile(models, sample, compile_model=True).to(DEV, BF).eval()
    eager = wc.compile(models, sample).to(DEV, BF).eval()
    x = torch.randn(b, n * t, d, device=DEV).to(BF)

    def check():
        y = graphed(x)
        assert len(graphed._graphs) == 1
        assert_lowp_close(y, _attn_oracle(graphed._orig_mod, x, n))
        eager.load_state_dict(graphed._orig_mod.state_dict())
        assert_lowp_close(y, eager(x).double())

    with torch.no_grad():
        check()
        check()
        a = graphed._orig_mod.stages['attn']
        a.q_weight.mul_(3.0)                                      # fused [q; kv] projection
        check()
        a.kv_bias.add_(0.5)
        check()
        new = {k: (v * 0.5 if k.endswith('kv_weight') else v) for k, v in graphed._orig_mod.state_dict().items()}
        graphed._orig_mod.load_state_dict(new)
        check()
        a.kv_weight.data.copy_(torch.randn_like(a.kv_weight) * 0.1)   # .data write
        y = graphed(x)
        assert_lowp_close(y, _attn_oracle(graphed._orig_mod, x, n))
    no_device_error()


# ---------------------------------------------------------------------------
# LSTM (the cfg4 recurrence, small)
# ---------------------------------------------------------------------------

class _Lstm(nn.Module):
    def __init__(self, i=16, h=32):
        super().__init__()
        self.lstm = nn.LSTM(i, h, batch_first=True)

    def forward(self, x):
        return self.lstm(x)[0]


def _lstm_oracle(wide, x, n):
    m = wide.stages['lstm']
    xn = O.packed_to_nfirst(x, n)
    bih, bhh = O.lstm_blocks(m.weight_ih.detach().cpu(), m.weight_hh.detach().cpu(), n)
    h4 = 4 * m.hidden_size
    out, _ = O.lstm(xn, None, None, bih, bhh, m.bias_ih.detach().cpu().view(n, h4),
                    m.bias_hh.detach().cpu().view(n, h4))
    return O.nfirst_to_packed(out)


def test_graphed_lstm_follows_parameter_updates():
    n, i, h, t, b = 4, 16, 32, 12, 3
    torch.manual_seed(14)
    models = [_Lstm(i, h) for _ in range(n)]
    sample = torch.randn(1, t, i)
    graphed = wc.compile(models, sample, compile_model=True).to(DEV)
    eager = wc.compile(models, sample).to(DEV)
    x = torch.randn(b, n * t, i, device=DEV)

    def check():
        y = graphed(x)
        assert len(graphed._graphs) == 1
        assert_fp32_close(y, _lstm_oracle(graphed._orig_mod, x, n))
        eager.load_state_dict(graphed._orig_mod.state_dict())
        assert_fp32_close(y, eager(x))

    with torch.no_grad():
        check()
        check()
        m = graphed._orig_mod.stages['lstm']
        m.weight_hh.mul_(1.5)                                     # diagonal blocks
        check()
        new = {k: (v * 0.75 if k.endswith('weight_ih') else v) for k, v in graphed._orig_mod.state_dict().items()}
        graphed._orig_mod.load_state_dict(new)
        check()
        m.weight_ih.data.mul_(-1.0)                               # .data write
        y = graphed(x)
        assert_fp32_close(y, _lstm_oracle(graphed._orig_mod, x, n))
    no_device_error()
