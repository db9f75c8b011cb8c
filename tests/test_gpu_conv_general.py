"""GPU parity of the tcgen05 per-tap conv kernel on the geometries beyond the
stride-1 2-D case: strides (TMA traversal steps), dilation, Conv3d, Conv1d,
channel counts that are not multiples of 64 (zero-padded K blocks) or of 16
(partial output tiles), with the fused epilogue and a packed input. Each
case first checks that the library picks the tensor-core kernel, then
compares with the oracle (bf16/f16 at rtol 2e-2 against an fp64
computation from the same rounded inputs and weights).
Reference primitives: wide_compiler/core/primitives/wide_conv1d.py:118-135,
wide_conv2d.py:169-194, wide_conv3d.py:102-125."""
import pytest
import torch

import wide_compiler as wc
from wide_compiler import ops
from gpu_util import assert_lowp_close, no_device_error
from oracle import wide_oracle as O

pytestmark = pytest.mark.gpu
DEV = 'cuda'
BF16, F16 = torch.bfloat16, torch.float16


def _case(n, b, cin, cout, sp, ks, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(n, b, cin, *sp, generator=gen).to(dtype)
    fan = cin
    for k in ks:
        fan *= k
    w = (torch.randn(n * cout, cin, *ks, generator=gen) / fan ** 0.5).to(dtype)
    bb = (torch.randn(n * cout, generator=gen) * 0.1).to(dtype)
    return x, w, bb


CASES = [
    # n, b, cin, cout, spatial, kernel, stride, padding, dilation, dtype
    (2, 2, 64, 64, (32, 32), (3, 3), (2, 2), (1, 1), (1, 1), BF16),
    (2, 3, 64, 128, (16, 16), (1, 1), (2, 2), (0, 0), (1, 1), BF16),
    (2, 1, 3, 64, (64, 64), (7, 7), (2, 2), (3, 3), (1, 1), BF16),
    (3, 2, 96, 64, (16, 16), (3, 3), (1, 1), (1, 1), (1, 1), F16),
    (2, 2, 64, 10, (12, 12), (3, 3), (1, 1), (1, 1), (1, 1), BF16),
    (2, 2, 32, 32, (6, 10, 10), (3, 3, 3), (1, 1, 1), (1, 1, 1), (1, 1, 1), BF16),
    (2, 1, 64, 64, (8, 16, 16), (3, 3, 3), (2, 2, 2), (1, 1, 1), (1, 1, 1), BF16),
    (2, 2, 16, 24, (5, 9, 7), (3, 1, 3), (1, 2, 1), (1, 0, 1), (2, 1, 1), F16),
    (3, 2, 32, 48, (100,), (5,), (2,), (2,), (1,), BF16),
    (2, 2, 64, 64, (17, 19), (3, 3), (2, 2), (2, 2), (2, 2), BF16),
    (2, 2, 64, 64, (20, 24), (3, 3), (2, 1), (1, 1), (1, 1), BF16),
    (1, 2, 8, 16, (33, 40), (5, 5), (3, 3), (2, 2), (1, 1), F16),
]


@pytest.mark.parametrize("n,b,cin,cout,sp,ks,st,pd,dl,dtype", CASES)
def test_conv_tensor_core_general(n, b, cin, cout, sp, ks, st, pd, dl, dtype):
    assert ops.conv_path(n, b, cin, cout, sp, ks, st, pd, dl, dtype) == ops.CONV_PATH_TAPS
    x, w, bb = _case(n, b, cin, cout, sp, ks, dtype, cin + cout + sum(sp) + sum(st))
    y = ops.conv_nd(x.to(DEV), w.to(DEV), bb.to(DEV), n, st, pd, dl)
    ref = O.conv_nd(x, w, bb, n, st, pd, dl)
    assert y.shape == ref.shape
    assert_lowp_close(y, ref)
    no_device_error()


@pytest.mark.parametrize("residual_first", [False, True])
def test_strided_conv_fused_epilogue(residual_first):
    """Bias, folded-BatchNorm scale/shift, ReLU and a residual fused into a
    stride-2 conv (TMA-stored output and TMA-loaded residual tiles)."""
    n, b, c = 2, 2, 64
    x, w, bb = _case(n, b, c, c, (32, 32), (3, 3), BF16, 11)
    gen = torch.Generator().manual_seed(12)
    sc = (torch.rand(n * c, generator=gen) + 0.5).to(BF16)
    sh = (torch.randn(n * c, generator=gen) * 0.1).to(BF16)
    res = torch.randn(n, b, c, 16, 16, generator=gen).to(BF16)
    y = ops.conv_nd(x.to(DEV), w.to(DEV), bb.to(DEV), n, (2, 2), (1, 1), (1, 1), scale=sc.to(DEV),
                    shift=sh.to(DEV), residual=res.to(DEV), act=ops.ACT_RELU, residual_first=residual_first)
    v = O.conv_nd(x, w, bb, n, (2, 2), (1, 1), (1, 1)) * sc.double().view(n, 1, c, 1, 1) + \
        sh.double().view(n, 1, c, 1, 1)
    ref = torch.clamp_min(v + res.double(), 0) if residual_first else torch.clamp_min(v, 0) + res.double()
    assert_lowp_close(y, ref)
    no_device_error()


def test_strided_conv_packed_input():
    """A packed [B, N*C, H, W] input (the TracedWideModel boundary) read by
    the staging of the strided tensor-core conv."""
    n, b, c = 3, 2, 64
    x, w, bb = _case(n, b, c, c, (16, 16), (3, 3), BF16, 21)
    packed = O.nfirst_to_packed(x).contiguous()
    y = ops.conv_nd(packed.to(DEV), w.to(DEV), bb.to(DEV), n, (2, 2), (1, 1), (1, 1),
                    in_layout=ops.LAYOUT_PACKED)
    assert y is not None
    assert_lowp_close(y, O.conv_nd(x, w, bb, n, (2, 2), (1, 1), (1, 1)))
    no_device_error()


def test_wide_conv3d_module_on_tensor_cores():
    """WideConv3d.from_modules (wide_conv3d.py:102-125) in bf16 runs on the
    tensor-core kernel and matches the per-model nn.Conv3d outputs."""
    torch.manual_seed(5)
    convs = [torch.nn.Conv3d(32, 32, 3, stride=(1, 2, 2), padding=1) for _ in range(3)]
    wide = wc.WideConv3d.from_modules(convs).to(DEV, BF16)
    x = torch.randn(3, 2, 32, 6, 12, 12).to(BF16)
    y = wide(x.to(DEV))
    for i, m in enumerate(convs):
        ref = O.conv_nd(x[i:i + 1], m.weight.detach().to(BF16), m.bias.detach().to(BF16), 1, (1, 2, 2), (1, 1, 1),
                        (1, 1, 1))
        assert_lowp_close(y[i:i + 1], ref)
    assert ops.conv_path(3, 2, 32, 32, (6, 12, 12), (3, 3, 3), (1, 2, 2), (1, 1, 1), (1, 1, 1), BF16) == \
        ops.CONV_PATH_TAPS
    no_device_error()


def test_strided_weight_cache_follows_updates():
    """The zero-padded packed weights (cin 3 -> one 64-channel block) are
    rebuilt after an in-place weight change."""
    n = 2
    x, w, bb = _case(n, 1, 3, 16, (20, 20), (3, 3), BF16, 31)
    wd, xd, bd = w.to(DEV), x.to(DEV), bb.to(DEV)
    y1 = ops.conv_nd(xd, wd, None, n, (2, 2), (1, 1), (1, 1))
    with torch.no_grad():
        wd.mul_(2.0)
    y2 = ops.conv_nd(xd, wd, None, n, (2, 2), (1, 1), (1, 1))
    assert_lowp_close(y2, 2 * y1.double())
    no_device_error()
