"""GPU parity of the halo-reuse convolution kernel (variant 0, where it
applies: 64-channel output tiles, output width a multiple of 8; variant 2,
its form with one shared halo buffer per 8 x 16 tile whose taps start at
row offsets inside the 128-byte swizzle pattern) and the per-tap kernel
(variant 1) against the float64 oracle, which restates the
reference's grouped conv (wide_compiler/core/primitives/wide_conv2d.py:169-194).
"""
import pytest
import torch

from wide_compiler import _native as N
from wide_compiler import ops
from gpu_util import assert_lowp_close, no_device_error
from oracle import wide_oracle as O

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def _case(n, b, cin, cout, sp, k, seed, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(seed)
    nd = len(sp)
    x = torch.randn(n, b, cin, *sp, generator=gen).to(dtype)
    fan = cin * k ** nd
    w = (torch.randn(n * cout, cin, *([k] * nd), generator=gen) / fan ** 0.5).to(dtype)
    bb = (torch.randn(n * cout, generator=gen) * 0.1).to(dtype)
    return x, w, bb


def _run(variant, *args, **kw):
    N.check(N.lib().widek_conv_set_variant(variant), "widek_conv_set_variant")
    try:
        y = ops.conv_nd(*args, **kw)
        torch.cuda.synchronize()
    finally:
        N.lib().widek_conv_set_variant(0)
    return y


SHAPES = [
    # n, b, cin, cout, spatial, k, pad, dil
    (3, 2, 64, 64, (32, 32), 3, 1, 1),      # cfg3's conv: tiles 16 x 8
    (2, 2, 64, 64, (8, 8), 3, 1, 1),        # tile width 8, one tile per image
    (2, 3, 64, 128, (13, 24), 3, 1, 1),     # two output tiles per pixel tile, ragged rows
    (2, 2, 128, 64, (10, 16), 3, 1, 1),     # two input-channel blocks
    (2, 2, 64, 64, (20, 40), 3, 2, 2),      # dilation 2: subtile rows = 8 + 4
    (2, 2, 64, 64, (9, 16), 3, 0, 1),       # no padding: output 7 x 14 is not a multiple of 8 -> per-tap
    (2, 2, 128, 128, (16, 16), 1, 0, 1),    # 1x1
    (2, 2, 64, 64, (1, 64), 3, 1, 1),       # a 1-row image (kernel rows past the image read zeros)
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "-".join(str(v) for v in s))
@pytest.mark.parametrize("variant", [0, 1, 2])
def test_conv_halo_vs_oracle(shape, variant):
    n, b, cin, cout, sp, k, p, d = shape
    x, w, bb = _case(n, b, cin, cout, sp, k, seed=sum(sp) + cin + k)
    nd = len(sp)
    y = _run(variant, x.to(DEV), w.to(DEV), bb.to(DEV), n, (1,) * nd, (p,) * nd, (d,) * nd)
    ref = O.conv_nd(x, w, bb, n, (1,) * nd, (p,) * nd, (d,) * nd)
    assert y.shape == ref.shape
    assert_lowp_close(y, ref)
    no_device_error()


@pytest.mark.parametrize("variant", [0, 2])
@pytest.mark.parametrize("residual_first", [False, True])
def test_conv_halo_fused_epilogue(residual_first, variant):
    """Folded BatchNorm scale/shift, ReLU and a residual, as the fused
    ResBlock convs use them, on the halo kernel."""
    n, b, c, hw = 2, 3, 64, 16
    x, w, bb = _case(n, b, c, c, (hw, hw), 3, seed=5)
    gen = torch.Generator().manual_seed(6)
    sc = (torch.rand(n * c, generator=gen) + 0.5).to(torch.bfloat16)
    sh = (torch.randn(n * c, generator=gen) * 0.1).to(torch.bfloat16)
    res = torch.randn(n, b, c, hw, hw, generator=gen).to(torch.bfloat16)
    y = _run(variant, x.to(DEV), w.to(DEV), bb.to(DEV), n, (1, 1), (1, 1), (1, 1), scale=sc.to(DEV),
             shift=sh.to(DEV), residual=res.to(DEV), act=ops.ACT_RELU, residual_first=residual_first)
    v = O.conv_nd(x, w, bb, n, (1, 1), (1, 1), (1, 1)) * sc.double().view(n, 1, c, 1, 1) + \
        sh.double().view(n, 1, c, 1, 1)
    if residual_first:
        ref = torch.relu(v + res.double())
    else:
        ref = torch.relu(v) + res.double()
    assert_lowp_close(y, ref)
    no_device_error()


def test_conv_halo_many_models_weight_reloads():
    """Enough models that each CTA's contiguous tile range crosses model
    boundaries (resident weights reloaded mid-range); checked per model on a
    sample against the per-tap kernel and on two models against the oracle."""
    n, b, c, hw = 40, 8, 64, 32
    x, w, bb = _case(n, b, c, c, (hw, hw), 3, seed=7)
    xd, wd, bd = x.to(DEV), w.to(DEV), bb.to(DEV)
    y0 = _run(0, xd, wd, bd, n, (1, 1), (1, 1), (1, 1))
    y1 = _run(1, xd, wd, bd, n, (1, 1), (1, 1), (1, 1))
    assert (y0.float() - y1.float()).abs().max().item() <= 2e-2 * y1.float().abs().max().item()
    for m in (0, n - 1):
        ref = O.conv_nd(x[m:m + 1], w[m * c:(m + 1) * c], bb[m * c:(m + 1) * c], 1, (1, 1), (1, 1), (1, 1))
        assert_lowp_close(y0[m:m + 1], ref)
    no_device_error()


@pytest.mark.parametrize("variant", [0, 2])
@pytest.mark.parametrize("ow", [8, 16, 24, 40])
def test_conv_halo_packed_residual_edges(ow, variant):
    """The halo kernel's TMA-stored packed output and TMA-loaded packed
    residual at ragged tile edges (rows past the image, a half-used
    16-pixel tile width)."""
    n, b, c, oh = 3, 2, 64, 19
    x, w, bb = _case(n, b, c, c, (oh, ow), 3, seed=ow)
    gen = torch.Generator().manual_seed(ow + 1)
    res = torch.randn(n, b, c, oh, ow, generator=gen).to(torch.bfloat16)
    pk = lambda t: t.transpose(0, 1).reshape(b, n * c, oh, ow).contiguous()
    y = _run(variant, x.to(DEV), w.to(DEV), bb.to(DEV), n, (1, 1), (1, 1), (1, 1), residual=pk(res).to(DEV),
             out_layout=ops.LAYOUT_PACKED, res_layout=ops.LAYOUT_PACKED)
    assert y is not None and y.shape == (b, n * c, oh, ow)
    ref = O.conv_nd(x, w, bb, n, (1, 1), (1, 1), (1, 1)) + res.double()
    assert_lowp_close(y.reshape(b, n, c, oh, ow).transpose(0, 1), ref)
    no_device_error()


@pytest.mark.parametrize("variant", [0, 2])
def test_conv_halo_channels_last_chain(variant):
    """conv1 -> conv2 as the fused ResBlock runs them: packed input, conv1
    writing channels-last (the 128-byte swizzled [pixel][channel] staging),
    conv2 reading it and adding the packed residual, packed output."""
    n, b, c, hw = 3, 2, 64, 32
    x, w1, b1 = _case(n, b, c, c, (hw, hw), 3, seed=41)
    _, w2, b2 = _case(n, b, c, c, (hw, hw), 3, seed=42)
    pk = lambda t: t.transpose(0, 1).reshape(b, n * c, hw, hw).contiguous()
    xp = pk(x).to(DEV)
    h = _run(variant, xp, w1.to(DEV), b1.to(DEV), n, (1, 1), (1, 1), (1, 1), act=ops.ACT_RELU,
             in_layout=ops.LAYOUT_PACKED, out_layout=ops.LAYOUT_CLAST)
    assert h is not None and h.shape == (n, b, hw, hw, c)
    y = _run(variant, h, w2.to(DEV), b2.to(DEV), n, (1, 1), (1, 1), (1, 1), residual=xp,
             in_layout=ops.LAYOUT_CLAST, out_layout=ops.LAYOUT_PACKED, res_layout=ops.LAYOUT_PACKED)
    h_ref = torch.relu(O.conv_nd(x, w1, b1, n, (1, 1), (1, 1), (1, 1))).to(torch.bfloat16)
    ref = O.conv_nd(h_ref, w2, b2, n, (1, 1), (1, 1), (1, 1)) + x.double()
    assert_lowp_close(y.reshape(b, n, c, hw, hw).transpose(0, 1), ref)
    no_device_error()
