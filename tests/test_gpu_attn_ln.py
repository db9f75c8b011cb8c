"""The attention output projection with the WideLayerNorm after it fused into
one launch (widek_linear_ln_fwd_ex: the GEMM's epilogue normalises each row
from the fp32 accumulator) against the fp64 oracle (oracle.linear, then
oracle.layernorm) at the bf16 tolerance, in the N-first and packed layouts,
and the TracedWideModel group that uses it (attention -> getitem ->
LayerNorm) against the oracle's attention + LayerNorm."""
import pytest
import torch
import torch.nn as nn

import wide_compiler as wc
from wide_compiler import ops
from gpu_util import assert_lowp_close, kernels_run, no_device_error
from oracle import wide_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


def _g(seed):
    return torch.Generator().manual_seed(seed)


def _case(n, b, t, k, o, dtype, bias, seed):
    x = torch.randn(n, b, t, k, generator=_g(seed)).to(dtype)
    w = (torch.randn(n, o, k, generator=_g(seed + 1)) / k ** 0.5).to(dtype)
    bb = (torch.randn(n, o, generator=_g(seed + 2)) * 0.5).to(dtype) if bias else None
    lw = torch.empty(n * o).uniform_(0.5, 1.5, generator=_g(seed + 3)).to(dtype)
    lb = (torch.randn(n * o, generator=_g(seed + 4)) * 0.1).to(dtype)
    return x, w, bb, lw, lb


def _ref(x, w, bb, lw, lb, eps):
    n, o = w.shape[0], w.shape[1]
    return O.layernorm(O.linear(x, w, bb), lw, lb, n, o, eps)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,b,t,k,o,bias", [
    (2, 2, 150, 512, 512, True),      # two MMAs of N = 256, a partial row tile
    (3, 1, 128, 64, 256, True),
    (1, 3, 40, 72, 48, False),        # o not a multiple of 32: the last 32-column chunk is clipped
    (2, 1, 300, 128, 400, True),      # second MMA of N = 144
    (4, 2, 64, 256, 16, True),
    (2, 2, 256, 512, 512, True),      # the cfg5 shape's row blocks (T a multiple of the 128-row tile)
])
@pytest.mark.parametrize("in_packed,out_packed", [(False, False), (True, True), (False, True)])
def test_linear_layernorm_fused_vs_oracle(dtype, n, b, t, k, o, bias, in_packed, out_packed):
    x, w, bb, lw, lb = _case(n, b, t, k, o, dtype, bias, seed=o + k)
    xin = O.nfirst_to_packed(x.reshape(n, b, t * k)).reshape(b, n * t, k) if in_packed else x
    xin = xin.contiguous().to(DEV)
    got = {}
    names = kernels_run(lambda: got.__setitem__('y', ops.linear_ln_layout(
        xin, w.to(DEV), None if bb is None else bb.to(DEV), lw.to(DEV), lb.to(DEV), 1e-5, in_packed, out_packed)))
    # packed rows are addressed per 128-row tile: with more than one row
    # block (B > 1), T must divide the tile or be a multiple of it (else the
    # call declines and launches nothing)
    fits = not (in_packed or out_packed) or b == 1 or t % 128 == 0 or 128 % t == 0
    if not fits:
        assert got['y'] is None and not any('linear_ln_kernel' in s for s in names), names
        return
    assert got['y'] is not None and any('linear_ln_kernel' in s for s in names), names
    ref = _ref(x, w, bb, lw, lb, 1e-5)                                 # [n, b, t, o]
    if out_packed:
        ref = O.nfirst_to_packed(ref.reshape(n, b, t * o)).reshape(b, n * t, o)
    assert_lowp_close(got['y'], ref)
    no_device_error()


def test_linear_layernorm_declines_unsupported_shapes():
    """o above 512, o not a multiple of 16 and fp32 are declined (None,
    nothing launched); the attention path then runs the two ops."""
    for o, dtype in [(520, torch.bfloat16), (40, torch.bfloat16), (64, torch.float32)]:
        x, w, bb, lw, lb = _case(1, 1, 8, 64, o, dtype, True, seed=1)
        assert ops.linear_ln_layout(x.to(DEV), w.to(DEV), bb.to(DEV), lw.to(DEV), lb.to(DEV), 1e-5,
                                    False, False) is None
    no_device_error()


class _AttnLN(nn.Module):
    def __init__(self, d, heads):
        super().__init__()
        self.attn = nn.MultiheadAttention(d, heads, batch_first=True)
        self.ln = nn.LayerNorm(d)

    def forward(self, x):
        a, _ = self.attn(x, x, x, need_weights=False)
        return self.ln(a)


@pytest.mark.parametrize("n,b,t,d,heads", [(3, 2, 128, 128, 2), (2, 1, 200, 512, 8)])
def test_traced_attention_layernorm_group(n, b, t, d, heads):
    """A TracedWideModel of N (MultiheadAttention -> LayerNorm) models runs
    the pair as one fused group: the packed input is read in place, the
    LayerNorm runs in the output projection's epilogue (no LayerNorm kernel
    launched), and the result matches the oracle's attention + LayerNorm.
    (T is a multiple of the 128-row tile, or B = 1, so that the packed rows
    fit the tensor-core kernels.)"""
    torch.manual_seed(0)
    models = [_AttnLN(d, heads).eval() for _ in range(n)]
    for m in models:
        with torch.no_grad():
            m.ln.weight.uniform_(0.5, 1.5)
            m.ln.bias.normal_(0, 0.1)
            m.attn.in_proj_bias.normal_(0, 0.1)
            m.attn.out_proj.bias.normal_(0, 0.1)
    wide = wc.compile(models, torch.randn(b, t, d), compile_model=False).to(DEV, torch.bfloat16)
    plan = wide._build_fusion_plan()
    assert [g['kind'] for g in plan['groups'].values()] == ['attn_ln']
    xs = [torch.randn(b, t, d, generator=_g(10 + i)).to(torch.bfloat16) for i in range(n)]
    packed = wc.pack_inputs([u.to(DEV) for u in xs])
    wide(packed)                       # first call: plan and derived weights
    got = {}
    names = kernels_run(lambda: got.__setitem__('y', wide(packed)))
    assert any('linear_ln_kernel' in s for s in names), names
    assert not any('layernorm' in s and 'bwd' not in s and 'linear_ln' not in s for s in names), names
    outs = wc.unpack_outputs(got['y'], n)
    for i, m in enumerate(models):
        a = m.attn
        w_in = a.in_proj_weight.detach().to(torch.bfloat16)[None]
        b_in = a.in_proj_bias.detach().to(torch.bfloat16)[None]
        xi = xs[i][None]
        y = O.attention(xi, xi, xi, w_in[:, :d], w_in[:, d:], b_in[:, :d], b_in[:, d:],
                        a.out_proj.weight.detach().to(torch.bfloat16)[None],
                        a.out_proj.bias.detach().to(torch.bfloat16)[None], heads)
        ref = O.layernorm(y, m.ln.weight.detach().to(torch.bfloat16), m.ln.bias.detach().to(torch.bfloat16), 1, d,
                          m.ln.eps)[0]
        assert_lowp_close(outs[i], ref)
    # the same graph node by node (no fusion) agrees with the fused run
    wide.fuse = False
    wide._fusion = None
    ref_unfused = wide(packed)
    assert_lowp_close(got['y'], ref_unfused.float())
    no_device_error()


def test_cfg5_bench_graph_sampled():
    """The cfg5 benchmark graph as bench.py builds it (TracedWideModel of
    attention -> LayerNorm models, T = 1024, d = 512, 8 heads, causal), at 2
    models: the fused group runs, and sampled (model, batch) outputs match
    the oracle's attention + LayerNorm."""
    import bench
    wl = bench.make_workload('cfg5', 2)
    wl._world_rank = (1, 0)
    wl._gather = False
    wl.setup(DEV, 0, 2, seed=1234)
    wl.step(wl.x)
    names = kernels_run(lambda: wl.step(wl.x))
    assert any('linear_ln_kernel' in s for s in names), names
    y = wl.step(wl.x)                                    # [B, 2*T, D] packed
    st = wl.module.local.stages
    a, ln = st['attn'], st['ln']
    b, t, d = wl.b, wl.t, wl.d
    xn = wl.x.view(b, 2, t, d).transpose(0, 1)           # [2, B, T, D]
    yn = y.view(b, 2, t, d).transpose(0, 1)
    for i, bi in [(0, 0), (1, 5)]:
        xi = xn[i, bi][None, None].cpu()
        sl = slice(i, i + 1)
        ref = O.attention(xi, xi, xi, a.q_weight[sl].cpu(), a.kv_weight[sl].cpu(), a.q_bias[sl].cpu(),
                          a.kv_bias[sl].cpu(), a.out_weight[sl].cpu(), a.out_bias[sl].cpu(), wl.heads,
                          is_causal=True)
        ref = O.layernorm(ref, ln.weight[i * d:(i + 1) * d].cpu(), ln.bias[i * d:(i + 1) * d].cpu(), 1, d, ln.eps)
        assert_lowp_close(yn[i, bi], ref[0, 0])
    no_device_error()
