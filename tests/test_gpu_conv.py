"""GPU parity: wide convolutions (tcgen05 implicit GEMM for bf16/f16, CUDA-core
direct kernel otherwise) against the reference fixtures and the oracle."""
import pytest
import torch

import wide_compiler as wc
from wide_compiler import ops
from conftest import golden_names, load_golden
from gpu_util import assert_fp32_close, assert_lowp_close, no_device_error
from oracle import wide_oracle as O
from test_api_host import _build_from_state

pytestmark = pytest.mark.gpu
DEV = 'cuda'


@pytest.mark.parametrize("name", golden_names('conv'))
def test_conv_golden(name):
    g = load_golden(name)
    mod = _build_from_state(g).to(DEV)
    assert_fp32_close(mod(g['inputs']['x'].to(DEV)), g['outputs']['y'])


def _conv_case(n, b, cin, cout, sp, k, dtype, seed, bias=True):
    gen = torch.Generator().manual_seed(seed)
    nd = len(sp)
    x = torch.randn(n, b, cin, *sp, generator=gen).to(dtype)
    fan = cin * k ** nd
    w = (torch.randn(n * cout, cin, *([k] * nd), generator=gen) / fan ** 0.5).to(dtype)
    bb = (torch.randn(n * cout, generator=gen) * 0.1).to(dtype) if bias else None
    return x, w, bb


@pytest.mark.parametrize("n,b,cin,cout,sp,k,p,d", [
    (3, 2, 64, 64, (32, 32), 3, 1, 1),
    (2, 3, 128, 128, (17, 20), 3, 2, 2),
    (2, 2, 64, 256, (8, 8), 1, 0, 1),
    (1, 1, 64, 16, (5, 200), 3, 1, 1),
    (2, 2, 64, 48, (7, 9), 3, 0, 1),
    (3, 2, 64, 32, (100,), 5, 2, 1),
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_conv_tensor_core(n, b, cin, cout, sp, k, p, d, dtype):
    x, w, bb = _conv_case(n, b, cin, cout, sp, k, dtype, n + cin + cout + k)
    nd = len(sp)
    y = ops.conv_nd(x.to(DEV), w.to(DEV), bb.to(DEV), n, (1,) * nd, (p,) * nd, (d,) * nd)
    ref = O.conv_nd(x, w, bb, n, (1,) * nd, (p,) * nd, (d,) * nd)
    assert y.shape == ref.shape
    assert_lowp_close(y, ref)
    no_device_error()


@pytest.mark.parametrize("n,b,cin,cout,sp,k,s,p,d,dtype", [
    (2, 2, 3, 8, (9, 11), 3, 2, 1, 1, torch.float32),
    (2, 2, 5, 4, (4, 5, 6), 3, 1, 1, 1, torch.float32),
    (2, 1, 4, 6, (33,), 4, 3, 2, 2, torch.float32),
    (2, 2, 64, 64, (40, 41), 3, 9, 1, 1, torch.bfloat16),   # stride > 8 (TMA step limit) -> CUDA cores
])
def test_conv_direct(n, b, cin, cout, sp, k, s, p, d, dtype):
    x, w, bb = _conv_case(n, b, cin, cout, sp, k, dtype, k + s + cin)
    nd = len(sp)
    assert ops.conv_path(n, b, cin, cout, sp, (k,) * nd, (s,) * nd, (p,) * nd, (d,) * nd, dtype) == \
        ops.CONV_PATH_DIRECT
    y = ops.conv_nd(x.to(DEV), w.to(DEV), bb.to(DEV), n, (s,) * nd, (p,) * nd, (d,) * nd)
    ref = O.conv_nd(x, w, bb, n, (s,) * nd, (p,) * nd, (d,) * nd)
    (assert_fp32_close if dtype == torch.float32 else assert_lowp_close)(y, ref)


@pytest.mark.parametrize("residual_first", [False, True])
def test_conv_fused_epilogue(residual_first):
    n, b, c = 2, 2, 64
    x, w, bb = _conv_case(n, b, c, c, (12, 12), 3, torch.bfloat16, 3)
    gen = torch.Generator().manual_seed(9)
    sc = (torch.rand(n * c, generator=gen) + 0.5).to(torch.bfloat16)
    sh = (torch.randn(n * c, generator=gen) * 0.1).to(torch.bfloat16)
    res = torch.randn(n, b, c, 12, 12, generator=gen).to(torch.bfloat16)
    y = ops.conv_nd(x.to(DEV), w.to(DEV), bb.to(DEV), n, (1, 1), (1, 1), (1, 1), scale=sc.to(DEV),
                    shift=sh.to(DEV), residual=res.to(DEV), act=ops.ACT_RELU, residual_first=residual_first)
    v = O.conv_nd(x, w, bb, n, (1, 1), (1, 1), (1, 1)) * sc.double().view(n, 1, c, 1, 1) + \
        sh.double().view(n, 1, c, 1, 1)
    if residual_first:
        ref = torch.clamp_min(v + res.double(), 0)
    else:
        ref = torch.clamp_min(v, 0) + res.double()
    assert_lowp_close(y, ref)


def test_conv_modules_and_weight_cache():
    torch.manual_seed(1)
    convs = [torch.nn.Conv2d(64, 64, 3, padding=1) for _ in range(3)]
    w = wc.WideConv2d.from_modules(convs, strategy='grouped').to(DEV, torch.bfloat16)
    x = torch.randn(3, 2, 64, 10, 10, device=DEV).to(torch.bfloat16)
    y1 = w(x)
    with torch.no_grad():
        w.grouped_conv.weight.mul_(2.0)     # version bump -> packed weights rebuilt
        w.grouped_conv.bias.mul_(2.0)
    y2 = w(x)
    assert_lowp_close(y2, 2 * y1.double())


def test_conv_cfg3_full_size_sampled():
    """Benchmark configuration cfg3 conv: N=100, B=32, 64->64, 3x3 pad 1, 32x32, bf16."""
    n, b, c = 100, 32, 64
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(n, b, c, 32, 32, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(n * c, c, 3, 3, device=DEV, generator=g) / 24).to(torch.bfloat16)
    bb = (torch.randn(n * c, device=DEV, generator=g) * 0.1).to(torch.bfloat16)
    y = ops.conv_nd(x, w, bb, n, (1, 1), (1, 1), (1, 1))
    for i, j in ((0, 0), (57, 31), (99, 5)):
        ref = O.conv_nd(x[i:i + 1, j:j + 1].cpu(), w[i * c:(i + 1) * c].cpu(), bb[i * c:(i + 1) * c].cpu(), 1,
                        (1, 1), (1, 1), (1, 1))
        assert_lowp_close(y[i:i + 1, j:j + 1], ref)
    no_device_error()


def test_traced_resblock_golden():
    g = load_golden('traced_resblock')
    n = g['meta']['n']
    import torch.nn as nn
    import torch.nn.functional as F

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

    models = []
    for i in range(n):
        m = ResBlock()
        m.load_state_dict({k.split('.', 1)[1]: v for k, v in g['state'].items() if k.startswith(f'm{i}.')})
        models.append(m.to(DEV).eval())
    wide = wc.compile(models, torch.randn(2, 4, 6, 6, device=DEV)).eval()
    out = wide(g['inputs']['packed'].to(DEV))
    assert_fp32_close(out, g['outputs']['y'])


class _RB(torch.nn.Module):
    def __init__(self, c, post_relu):
        super().__init__()
        self.post_relu = post_relu
        self.conv1 = torch.nn.Conv2d(c, c, 3, padding=1)
        self.bn1 = torch.nn.BatchNorm2d(c)
        self.conv2 = torch.nn.Conv2d(c, c, 3, padding=1)
        self.bn2 = torch.nn.BatchNorm2d(c)

    def forward(self, x):
        h = torch.nn.functional.relu(self.bn1(self.conv1(x)))
        y = self.bn2(self.conv2(h)) + x
        return torch.nn.functional.relu(y) if self.post_relu else y


@pytest.mark.parametrize("post_relu", [False, True])
def test_traced_resblock_fused_matches_unfused_bf16(post_relu):
    torch.manual_seed(2)
    n, c = 3, 64
    models = []
    for _ in range(n):
        m = _RB(c, post_relu)
        with torch.no_grad():
            for bn in (m.bn1, m.bn2):
                bn.running_mean.normal_(0, 1)
                bn.running_var.uniform_(0.5, 2.0)
                bn.weight.uniform_(0.5, 1.5)
                bn.bias.normal_(0, 0.1)
        models.append(m.to(DEV, torch.bfloat16).eval())
    wide = wc.compile(models, torch.randn(2, c, 16, 16, device=DEV, dtype=torch.bfloat16)).eval()
    x = torch.randn(2, n * c, 16, 16, device=DEV).to(torch.bfloat16)
    y_fused = wide(x)
    assert wide._fusion['groups'], "expected fused groups"
    wide.fuse = False
    wide._fusion = None
    y_plain = wide(x)
    assert_lowp_close(y_fused, y_plain.double())
    # and against the per-model torch modules in fp32
    xs = wc.unpack(x, n)
    ref = torch.cat([models[i].float()(xs[i].float()) for i in range(n)], dim=1)
    assert_lowp_close(y_fused, ref.double(), rtol=5e-2)


def test_traced_fused_bn_follows_in_place_changes():
    """The fused conv groups keep the folded BatchNorm between forwards; an
    in-place change of its statistics or affine parameters, or a replaced
    tensor, must show in the next forward."""
    torch.manual_seed(4)
    n, c = 2, 64
    models = [_RB(c, False).to(DEV, torch.bfloat16).eval() for _ in range(n)]
    wide = wc.compile(models, torch.randn(2, c, 16, 16, device=DEV, dtype=torch.bfloat16)).eval()
    x = torch.randn(2, n * c, 16, 16, device=DEV).to(torch.bfloat16)

    def ref():                                    # the N modules in fp32 (converted in place)
        xs = wc.unpack(x, n)
        return torch.cat([models[i].float()(xs[i].float()) for i in range(n)], dim=1).double()

    with torch.no_grad():
        assert_lowp_close(wide(x), ref(), rtol=5e-2)
        assert wide._fusion['groups'], "expected fused groups"
        wide(x)                                   # second forward: folded values reused
        bn = wide.stages['bn1'].op
        bn.running_mean.add_(0.5)                 # in place
        bn.weight.mul_(1.5)
        for i, m in enumerate(models):            # the same change in the references
            m.bn1.running_mean.copy_(bn.running_mean[i * c:(i + 1) * c].to(torch.bfloat16))
            m.bn1.weight.copy_(bn.weight[i * c:(i + 1) * c].to(torch.bfloat16))
        assert_lowp_close(wide(x), ref(), rtol=5e-2)
        bn2 = wide.stages['bn2'].op
        bn2.running_var = bn2.running_var * 2.0   # replaced tensor
        for i, m in enumerate(models):
            m.bn2.running_var.copy_(bn2.running_var[i * c:(i + 1) * c].to(torch.bfloat16))
        assert_lowp_close(wide(x), ref(), rtol=5e-2)
    no_device_error()


def test_traced_fusion_falls_back_in_training_mode():
    torch.manual_seed(3)
    models = [_RB(8, False).to(DEV) for _ in range(2)]
    wide = wc.compile(models, torch.randn(2, 8, 6, 6, device=DEV))
    wide.train()
    x = torch.randn(4, 16, 6, 6, device=DEV)
    y = wide(x)          # BatchNorm in training mode: groups run node by node
    for m in models:
        m.train()
    xs = wc.unpack(x, 2)
    ref = torch.cat([models[i](xs[i]) for i in range(2)], dim=1)
    assert_fp32_close(y, ref.detach())
