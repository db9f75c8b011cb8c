"""GPU parity of the layout-fused convolution entry (widek_conv_fwd_ex):
packed [B, N*C, H, W] inputs / outputs / residuals and channels-last
[N, B, H, W, C] intermediates, against the float64 oracle of the reference's
grouped conv (wide_compiler/core/primitives/wide_conv2d.py:169-194) and its
TracedWideModel boundary pack/unpack (core/traced_wide.py:463-469, :531-532).
"""
import pytest
import torch

import wide_compiler as wc
from wide_compiler import ops
from gpu_util import assert_lowp_close, no_device_error
from oracle import wide_oracle as O

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def _case(n, b, c, hw, seed):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(n, b, c, hw, hw, generator=gen).to(torch.bfloat16)
    w = (torch.randn(n * c, c, 3, 3, generator=gen) / (c * 9) ** 0.5).to(torch.bfloat16)
    bb = (torch.randn(n * c, generator=gen) * 0.1).to(torch.bfloat16)
    sc = (torch.rand(n * c, generator=gen) + 0.5).to(torch.bfloat16)
    sh = (torch.randn(n * c, generator=gen) * 0.1).to(torch.bfloat16)
    return x, w, bb, sc, sh


def _packed(t):       # [N, B, C, H, W] -> [B, N*C, H, W]
    n, b, c = t.shape[:3]
    return t.transpose(0, 1).reshape(b, n * c, *t.shape[3:]).contiguous()


def _clast(t):        # [N, B, C, H, W] -> [N, B, H, W, C]
    return t.permute(0, 1, 3, 4, 2).contiguous()


def _from_packed(t, n):
    b, nc = t.shape[:2]
    return t.reshape(b, n, nc // n, *t.shape[2:]).transpose(0, 1)


def _from_clast(t):
    return t.permute(0, 1, 4, 2, 3)


def test_packed_in_clast_out_then_clast_in_packed_out():
    """A ResBlock-shaped chain in the fused layouts: conv1 reads the packed
    input and writes channels-last (BN + ReLU fused); conv2 reads that, adds
    the packed input as residual (BN, then add) and writes the packed output."""
    n, b, c, hw = 3, 2, 64, 32
    x, w1, b1, s1, h1 = _case(n, b, c, hw, 1)
    _, w2, b2, s2, h2 = _case(n, b, c, hw, 2)
    xp = _packed(x).to(DEV)
    y1 = ops.conv_nd(xp, w1.to(DEV), b1.to(DEV), n, (1, 1), (1, 1), (1, 1), scale=s1.to(DEV), shift=h1.to(DEV),
                     act=ops.ACT_RELU, in_layout=ops.LAYOUT_PACKED, out_layout=ops.LAYOUT_CLAST)
    assert y1 is not None and y1.shape == (n, b, hw, hw, c)
    ref1 = torch.relu(O.conv_nd(x, w1, b1, n, (1, 1), (1, 1), (1, 1)) * s1.double().view(n, 1, c, 1, 1) +
                      h1.double().view(n, 1, c, 1, 1))
    assert_lowp_close(_from_clast(y1), ref1)
    y2 = ops.conv_nd(y1, w2.to(DEV), b2.to(DEV), n, (1, 1), (1, 1), (1, 1), scale=s2.to(DEV), shift=h2.to(DEV),
                     residual=xp, in_layout=ops.LAYOUT_CLAST, out_layout=ops.LAYOUT_PACKED,
                     res_layout=ops.LAYOUT_PACKED)
    assert y2 is not None and y2.shape == (b, n * c, hw, hw)
    # reference for conv2 from the GPU's own conv1 output (rounded as stored)
    h_in = _from_clast(y1).float().cpu().to(torch.bfloat16).contiguous()
    ref2 = O.conv_nd(h_in, w2, b2, n, (1, 1), (1, 1), (1, 1)) * s2.double().view(n, 1, c, 1, 1) + \
        h2.double().view(n, 1, c, 1, 1) + x.double()
    assert_lowp_close(_from_packed(y2, n), ref2)
    no_device_error()


@pytest.mark.parametrize("in_l,out_l", [(1, 0), (2, 0), (0, 1), (0, 2), (2, 2), (1, 1)])
def test_layout_pairs(in_l, out_l):
    n, b, c, hw = 2, 3, 64, 16
    x, w, bb, _, _ = _case(n, b, c, hw, 10 + 3 * in_l + out_l)
    xin = {0: x, 1: _packed(x), 2: _clast(x)}[in_l].to(DEV)
    y = ops.conv_nd(xin, w.to(DEV), bb.to(DEV), n, (1, 1), (1, 1), (1, 1), in_layout=in_l, out_layout=out_l)
    assert y is not None
    y = {0: lambda t: t, 1: lambda t: _from_packed(t, n), 2: _from_clast}[out_l](y)
    assert_lowp_close(y, O.conv_nd(x, w, bb, n, (1, 1), (1, 1), (1, 1)))
    no_device_error()


def test_unsupported_layout_returns_none():
    """A channels-last output with a residual is not offered: the call
    returns None and launches nothing."""
    n, b, c, hw = 2, 2, 64, 16
    x, w, bb, _, _ = _case(n, b, c, hw, 3)
    y = ops.conv_nd(x.to(DEV), w.to(DEV), bb.to(DEV), n, (1, 1), (1, 1), (1, 1), residual=x.to(DEV),
                    out_layout=ops.LAYOUT_CLAST)
    assert y is None
    no_device_error()


def test_traced_resblock_fused_layouts_match_unfused():
    """The TracedWideModel ResBlock (packed in, packed out) with fusion on
    (layout-fused convs) equals the node-by-node run of the same model."""
    import torch.nn as nn

    class Block(nn.Module):
        def __init__(self, c):
            super().__init__()
            self.c1 = nn.Conv2d(c, c, 3, padding=1)
            self.b1 = nn.BatchNorm2d(c)
            self.c2 = nn.Conv2d(c, c, 3, padding=1)
            self.b2 = nn.BatchNorm2d(c)

        def forward(self, x):
            h = torch.relu(self.b1(self.c1(x)))
            return self.b2(self.c2(h)) + x

    torch.manual_seed(4)
    n, b, c, hw = 4, 3, 64, 16
    blocks = [Block(c) for _ in range(n)]
    for blk in blocks:
        for bn in (blk.b1, blk.b2):
            bn.running_mean.normal_(0, 0.1)
            bn.running_var.uniform_(0.5, 1.5)
    model = wc.compile(blocks, torch.randn(1, c, hw, hw)).to(DEV, torch.bfloat16).eval()
    x = torch.randn(b, n * c, hw, hw, device=DEV).to(torch.bfloat16)
    y_fused = model(x)
    model.fuse = False
    model._fusion = None
    y_plain = model(x)
    assert y_fused.shape == y_plain.shape == (b, n * c, hw, hw)
    assert_lowp_close(y_fused, y_plain.double())
    no_device_error()
