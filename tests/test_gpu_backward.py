"""Backward kernels (csrc/backward.cu) against the oracle's gradient formulas.

The oracle's formulas (oracle/wide_oracle.py linear_grads / layernorm_grads)
are pinned to the reference's own autograd by the grad_* golden fixtures
(tests/test_oracle_golden.py). Here the kernels run through the public
autograd path (the wide modules and ops with requires_grad) and through the
C-ABI wrappers directly: fp32 within rtol 1e-3 / atol 1e-4, bf16 within
rtol 2e-2 of the fp64 oracle evaluated on the same (rounded) inputs; the
byte-moving transpose is bit-exact.
"""
import pytest
import torch
import torch.nn as nn

import wide_compiler as wc
from wide_compiler import ops
from conftest import golden_names, load_golden
from gpu_util import assert_fp32_close, assert_lowp_close, kernels_run, no_device_error
from oracle import wide_oracle as O
from test_api_host import _build_from_state

pytestmark = [pytest.mark.gpu, pytest.mark.grad]
DEV = torch.device('cuda', 0)
ACTS = {'none': ops.ACT_NONE, 'relu': ops.ACT_RELU, 'gelu': ops.ACT_GELU}


def _close(dtype, a, e):
    (assert_fp32_close if dtype == torch.float32 else assert_lowp_close)(a, e)


def _g(seed):
    return torch.Generator().manual_seed(seed)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("b,r,c", [(3, 64, 64), (2, 100, 72), (5, 17, 33), (1, 1, 129), (4, 256, 8), (2, 130, 260)])
@pytest.mark.parametrize("offset", [0, 1])
def test_transpose_bit_exact(dtype, b, r, c, offset):
    """[b, r, c] -> [b, c, r]; offset 1 starts the tensors one element past
    a 16-byte boundary, which takes the element-wise paths."""
    x = torch.randn(b, r, c, generator=_g(r * c)).to(dtype)
    buf = torch.empty(b * r * c + offset, dtype=dtype, device=DEV)
    xd = buf[offset:].view(b, r, c)
    xd.copy_(x)
    y = ops.transpose(xd)
    assert torch.equal(y.cpu(), x.transpose(1, 2).contiguous())
    no_device_error()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,shape,k,o,bias,act", [
    (3, (40,), 64, 96, True, 'none'),
    (2, (17,), 20, 12, True, 'relu'),              # ragged: CUDA-core GEMMs, element-wise transposes
    (4, (256,), 128, 256, False, 'gelu'),
    (2, (3, 11), 72, 40, True, 'gelu'),            # extra batch dims
    (5, (1,), 8, 16, True, 'relu'),
    (2, (300,), 136, 520, True, 'none'),           # several M / N tiles, ragged K blocks (MN-major path)
    (1, (1000,), 64, 64, False, 'none'),           # dW reduces over 1000 rows (16 K blocks)
])
def test_linear_backward_vs_oracle(dtype, n, shape, k, o, bias, act):
    x = torch.randn(n, *shape, k, generator=_g(k)).to(dtype)
    w = (torch.randn(n, o, k, generator=_g(o)) / k ** 0.5).to(dtype)
    b = (torch.randn(n, o, generator=_g(3)) * 0.1).to(dtype) if bias else None
    dy = torch.randn(n, *shape, o, generator=_g(5)).to(dtype)
    xg = x.to(DEV).requires_grad_()
    wg = w.to(DEV).requires_grad_()
    bg = b.to(DEV).requires_grad_() if bias else None
    y = ops.linear(xg, wg, bg, ACTS[act])
    names = kernels_run(lambda: y.backward(dy.to(DEV)))
    # bf16 with 16-byte rows: the tcgen05 GEMM reads W, dY and x MN-major (no
    # transposes); otherwise transposed copies feed the forward's GEMM
    mn = dtype == torch.bfloat16 and o % 8 == 0 and k % 8 == 0
    assert any('transpose_kernel' in s for s in names) == (not mn), names
    if mn:
        assert any('linear_tc_kernel' in s for s in names), names
    rdx, rdw, rdb = O.linear_grads(x, w, b, dy, act)
    _close(dtype, xg.grad, rdx)
    _close(dtype, wg.grad, rdw)
    if bias:
        _close(dtype, bg.grad, rdb)
    no_device_error()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_linear_backward_partial_and_empty(dtype):
    """Only the asked gradients are computed; zero rows give zero dW / db."""
    n, m, k, o = 3, 24, 32, 16
    x = torch.randn(n, m, k, generator=_g(1)).to(dtype)
    w = torch.randn(n, o, k, generator=_g(2)).to(dtype)
    dy = torch.randn(n, m, o, generator=_g(3)).to(dtype)
    dx, dw, db = ops.linear_bwd(x.to(DEV), w.to(DEV), dy.to(DEV), True, False, False)
    assert dw is None and db is None
    _close(dtype, dx, O.linear_grads(x, w, None, dy)[0])
    z = torch.empty(n, 0, k, dtype=dtype, device=DEV)
    dx, dw, db = ops.linear_bwd(z, w.to(DEV), torch.empty(n, 0, o, dtype=dtype, device=DEV))
    assert dx.shape == (n, 0, k) and float(dw.abs().sum()) == 0.0 and float(db.abs().sum()) == 0.0
    no_device_error()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,rows,d", [
    (3, (4, 6), 40), (2, (37,), 100), (4, (8, 16), 512), (2, (5,), 1024), (3, (7,), 768), (2, (3000,), 256),
    (1, (1,), 1),
])
def test_layernorm_backward_vs_oracle(dtype, n, rows, d):
    x = (torch.randn(n, *rows, d, generator=_g(d)) * 2 + 0.5).to(dtype)
    w = torch.empty(n * d).uniform_(0.5, 1.5, generator=_g(1)).to(dtype)
    b = (torch.randn(n * d, generator=_g(2)) * 0.1).to(dtype)
    dy = torch.randn(n, *rows, d, generator=_g(3)).to(dtype)
    xg, wg, bg = (t.to(DEV).requires_grad_() for t in (x, w, b))
    y = ops.layernorm(xg, wg, bg, n, d, 1e-5)
    names = kernels_run(lambda: y.backward(dy.to(DEV)))
    assert any('layernorm_bwd_kernel' in s for s in names), names
    rdx, rdw, rdb = O.layernorm_grads(x, w, dy, n, d, 1e-5)
    _close(dtype, xg.grad, rdx)
    _close(dtype, wg.grad, rdw)
    _close(dtype, bg.grad, rdb)
    no_device_error()


@pytest.mark.parametrize("name", golden_names('grad_linear') + golden_names('grad_layernorm')
                         + golden_names('grad_batchnorm') + golden_names('grad_groupnorm'))
def test_golden_gradients_through_modules(name):
    """The reference's own gradients (grad_* fixtures) reproduced through
    this package's modules (WideLinear + activation glue, WideLayerNorm,
    WideBatchNorm2d in training and eval mode, WideGroupNorm)."""
    g = load_golden(name)
    mod = _build_from_state(g).to(DEV)
    if g['kind'] == 'grad_batchnorm':
        mod.train(g['meta']['train'])
    x = g['inputs']['x'].to(DEV).requires_grad_()
    y = mod(x)
    if g['kind'] == 'grad_linear' and g['meta']['act'] != 'none':
        y = ops.unary(y, g['meta']['act'])
    assert_fp32_close(y.detach(), g['outputs']['y'])
    y.backward(g['inputs']['dy'].to(DEV))
    want = g['outputs']['grads']
    assert_fp32_close(x.grad, want['x'])
    for key, p in mod.named_parameters():
        assert_fp32_close(p.grad, want[key])
    no_device_error()


class _MLP(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(64, 128)
        self.fc2 = nn.Linear(128, 64)

    def forward(self, x):
        return self.fc2(torch.relu(self.fc1(x)))


def test_traced_mlp_training_step_gradients():
    """A TracedWideModel of N MLPs (cfg1's shape) trained one step: the
    gradients of every model's parameters equal those of the stand-alone
    models (fp64 autograd on the CPU), and the backward runs on the
    library's kernels."""
    n, b = 6, 32
    torch.manual_seed(0)
    models = [_MLP() for _ in range(n)]
    wide = wc.compile(models, torch.randn(b, 64), compile_model=False).to(DEV)
    xs = [torch.randn(b, 64, generator=_g(10 + i)) for i in range(n)]
    dys = [torch.randn(b, 64, generator=_g(50 + i)) for i in range(n)]
    packed = wc.pack_inputs([t.to(DEV) for t in xs])
    y = wide(packed)
    dy_packed = wc.pack_inputs([t.to(DEV) for t in dys])
    names = kernels_run(lambda: y.backward(dy_packed))
    assert any('transpose_kernel' in s for s in names) and any('act_bwd_kernel' in s for s in names), names
    grads = {k: p.grad for k, p in wide.named_parameters()}
    assert all(v is not None for v in grads.values())
    for i, (m, xi, dyi) in enumerate(zip(models, xs, dys)):
        md = _MLP().double()
        md.load_state_dict(m.state_dict())
        md(xi.double()).backward(dyi.double())
        for key, p in md.named_parameters():
            assert_fp32_close(grads[f'stages.{key}'][i], p.grad)
    no_device_error()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,b,c,sp,batch_stats,affine", [
    (3, 5, 4, (6, 7), True, True),
    (2, 32, 64, (32, 32), True, True),        # cfg3's BatchNorm size per model (vector path)
    (3, 4, 6, (5, 5), False, True),           # eval mode: running statistics
    (2, 3, 5, (7,), True, False),             # 1-d, no affine, element-wise path (L = 7)
])
def test_batchnorm_backward_vs_oracle(dtype, n, b, c, sp, batch_stats, affine):
    x = (torch.randn(n, b, c, *sp, generator=_g(c)) * 1.5 + 0.3).to(dtype)
    w = torch.empty(n * c).uniform_(0.5, 1.5, generator=_g(1)).to(dtype) if affine else None
    bb = (torch.randn(n * c, generator=_g(2)) * 0.1).to(dtype) if affine else None
    rm = torch.randn(n * c, generator=_g(3)).to(dtype)
    rv = torch.empty(n * c).uniform_(0.5, 2.0, generator=_g(4)).to(dtype)
    dy = torch.randn(n, b, c, *sp, generator=_g(5)).to(dtype)
    xg = x.to(DEV).requires_grad_()
    wg = w.to(DEV).requires_grad_() if affine else None
    bg = bb.to(DEV).requires_grad_() if affine else None
    rmd, rvd = rm.to(DEV), rv.to(DEV)
    y = ops.batchnorm(xg, n, c, wg, bg, rmd, rvd, batch_stats, False, 0.1, 1e-5)
    names = kernels_run(lambda: y.backward(dy.to(DEV)))
    assert any('norm_bwd_kernel' in s for s in names), names
    rdx, rdw, rdb = O.batchnorm_grads(x, n, c, w, rm, rv, dy, batch_stats, 1e-5)
    _close(dtype, xg.grad, rdx)
    if affine:
        _close(dtype, wg.grad, rdw)
        _close(dtype, bg.grad, rdb)
    no_device_error()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,b,c,groups,sp,affine", [
    (3, 2, 8, 4, (5, 6), True),
    (2, 4, 64, 32, (16, 16), True),           # vector path, two channels per group
    (2, 3, 6, 6, (7,), False),                # InstanceNorm (one channel per group), element-wise path
    (1, 2, 12, 1, (8, 8), True),              # one group: the whole sample
])
def test_groupnorm_backward_vs_oracle(dtype, n, b, c, groups, sp, affine):
    x = (torch.randn(n, b, c, *sp, generator=_g(c + groups)) * 2 + 0.5).to(dtype)
    w = torch.empty(n * c).uniform_(0.5, 1.5, generator=_g(1)).to(dtype) if affine else None
    bb = (torch.randn(n * c, generator=_g(2)) * 0.1).to(dtype) if affine else None
    dy = torch.randn(n, b, c, *sp, generator=_g(5)).to(dtype)
    xg = x.to(DEV).requires_grad_()
    wg = w.to(DEV).requires_grad_() if affine else None
    bg = bb.to(DEV).requires_grad_() if affine else None
    y = ops.groupnorm(xg, n, groups, wg, bg, 1e-5)
    names = kernels_run(lambda: y.backward(dy.to(DEV)))
    assert any('norm_bwd_kernel' in s for s in names), names
    rdx, rdw, rdb = O.groupnorm_grads(x, n, groups, w, dy, 1e-5)
    _close(dtype, xg.grad, rdx)
    if affine:
        _close(dtype, wg.grad, rdw)
        _close(dtype, bg.grad, rdb)
    no_device_error()
