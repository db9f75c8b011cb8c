"""GPU parity: WideBatchNorm1d/2d (eval + train with running-stat update),
WideGroupNorm, WideInstanceNorm1d/2d and WideEmbedding, against the reference
fixtures and the oracle."""
import pytest
import torch

import wide_compiler as wc
from wide_compiler import _native, ops
from conftest import golden_names, load_golden
from gpu_util import assert_fp32_close, assert_lowp_close, no_device_error
from oracle import wide_oracle as O
from test_api_host import _build_from_state

pytestmark = pytest.mark.gpu
DEV = 'cuda'


@pytest.mark.parametrize("name", golden_names('batchnorm'))
def test_batchnorm_golden(name):
    g = load_golden(name)
    mod = _build_from_state(g).to(DEV)
    mod.train(g['meta']['train'])
    y = mod(g['inputs']['x'].to(DEV))
    assert_fp32_close(y, g['outputs']['y'])
    if g['meta']['train']:
        assert_fp32_close(mod.op.running_mean, g['outputs']['running_mean'])
        assert_fp32_close(mod.op.running_var, g['outputs']['running_var'])
        assert int(mod.op.num_batches_tracked) == int(g['outputs']['num_batches_tracked'])


@pytest.mark.parametrize("name", golden_names('groupnorm') + golden_names('instancenorm') + golden_names('embedding'))
def test_groupnorm_instancenorm_embedding_golden(name):
    g = load_golden(name)
    mod = _build_from_state(g).to(DEV)
    x = g['inputs']['idx' if g['kind'] == 'embedding' else 'x'].to(DEV)
    assert_fp32_close(mod(x), g['outputs']['y'])


def _bn_params(n, c, dtype, gen):
    w = (torch.rand(n * c, generator=gen) + 0.5).to(dtype)
    b = (torch.randn(n * c, generator=gen) * 0.1).to(dtype)
    rm = torch.randn(n * c, generator=gen).to(dtype)
    rv = (torch.rand(n * c, generator=gen) * 1.5 + 0.5).to(dtype)
    return w, b, rm, rv


@pytest.mark.parametrize("shape", [(16, 8, 64, 32, 32), (3, 5, 7, 9), (4, 6, 10), (2, 64, 3, 33, 17)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_batchnorm_eval_random(shape, dtype):
    gen = torch.Generator().manual_seed(sum(shape))
    n, c = shape[0], shape[2]
    x = (torch.randn(*shape, generator=gen) * 2 + 0.5).to(dtype)
    w, b, rm, rv = _bn_params(n, c, dtype, gen)
    y = ops.batchnorm(x.to(DEV), n, c, w.to(DEV), b.to(DEV), rm.to(DEV), rv.to(DEV), use_batch_stats=False,
                      update_running=False, momentum=0.0, eps=1e-5)
    ref, _, _ = O.batchnorm(x, n, c, w, b, rm, rv, False)
    (assert_fp32_close if dtype == torch.float32 else assert_lowp_close)(y, ref)


@pytest.mark.parametrize("shape", [(2, 64, 3, 33, 17), (3, 32, 8, 64, 64), (4, 6, 10), (1, 1000, 4, 50),
                                   # one-pass kernel: 16-byte vectors (up to 8 per thread), scalars
                                   (4, 32, 8, 32, 32), (3, 16, 5, 16, 16), (5, 3, 4, 8), (2, 7, 3, 5, 3)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_batchnorm_train_random(shape, dtype):
    gen = torch.Generator().manual_seed(sum(shape) + 1)
    n, c = shape[0], shape[2]
    x = (torch.randn(*shape, generator=gen) * 1.5 + 3.0).to(dtype)
    w, b, rm, rv = _bn_params(n, c, dtype, gen)
    rm_d, rv_d = rm.to(DEV), rv.to(DEV)
    y = ops.batchnorm(x.to(DEV), n, c, w.to(DEV), b.to(DEV), rm_d, rv_d, use_batch_stats=True,
                      update_running=True, momentum=0.1, eps=1e-5)
    ref, new_rm, new_rv = O.batchnorm(x, n, c, w, b, rm, rv, True, momentum=0.1)
    close = assert_fp32_close if dtype == torch.float32 else assert_lowp_close
    close(y, ref)
    close(rm_d, new_rm)
    close(rv_d, new_rv)


def test_batchnorm_module_momentum_none_and_no_affine():
    bns = [torch.nn.BatchNorm2d(5, momentum=None, affine=False) for _ in range(3)]
    w = wc.WideBatchNorm2d.from_modules(bns).to(DEV).train()
    x = torch.randn(3, 4, 5, 6, 6)
    for step in range(2):
        y = w(x.to(DEV) + step)
    # cumulative average over 2 batches
    rm = torch.zeros(15, dtype=torch.float64)
    rv = torch.ones(15, dtype=torch.float64)
    for step in range(2):
        _, rm, rv = O.batchnorm(x + step, 3, 5, None, None, rm, rv, True, momentum=1.0 / (step + 1))
    assert_fp32_close(w.op.running_mean, rm)
    assert_fp32_close(w.op.running_var, rv)
    assert int(w.op.num_batches_tracked) == 2


@pytest.mark.parametrize("shape,groups", [((4, 8, 64, 32, 32), 8), ((3, 2, 12, 7, 5), 3), ((2, 3, 16, 300, 300), 2),
                                          ((5, 4, 6, 33), 6), ((2, 2, 8), 4)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_groupnorm_random(shape, groups, dtype):
    gen = torch.Generator().manual_seed(groups + sum(shape))
    n, c = shape[0], shape[2]
    x = (torch.randn(*shape, generator=gen) * 2 - 1).to(dtype)
    w = (torch.rand(n * c, generator=gen) + 0.5).to(dtype)
    b = (torch.randn(n * c, generator=gen) * 0.1).to(dtype)
    y = ops.groupnorm(x.to(DEV), n, groups, w.to(DEV), b.to(DEV), 1e-5)
    ref = O.groupnorm(x, n, groups, w, b, 1e-5)
    (assert_fp32_close if dtype == torch.float32 else assert_lowp_close)(y, ref)


def test_instancenorm_modes():
    ins = [torch.nn.InstanceNorm2d(4, affine=True, track_running_stats=True) for _ in range(3)]
    wide = wc.WideInstanceNorm2d.from_modules(ins).to(DEV)
    x = torch.randn(3, 5, 4, 6, 7)
    wide.train()
    y = wide(x.to(DEV))
    assert_fp32_close(y, O.groupnorm(x, 3, 4, wide.norm.weight.detach().cpu(), wide.norm.bias.detach().cpu(), 1e-5))
    # torch reference for the running-stat update on the channel-packed tensor
    ref_in = torch.nn.InstanceNorm2d(12, affine=True, track_running_stats=True).train()
    ref_in(x.permute(1, 0, 2, 3, 4).reshape(5, 12, 6, 7))
    assert_fp32_close(wide.norm.running_mean, ref_in.running_mean)
    assert_fp32_close(wide.norm.running_var, ref_in.running_var)
    wide.eval()
    ye = wide(x.to(DEV))
    ref, _, _ = O.batchnorm(x, 3, 4, wide.norm.weight.detach().cpu(), wide.norm.bias.detach().cpu(),
                            wide.norm.running_mean.cpu(), wide.norm.running_var.cpu(), False)
    assert_fp32_close(ye, ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_embedding_random(dtype):
    n, v, d = 5, 100, 24
    wt = torch.randn(n, v, d).to(dtype)
    idx = torch.randint(-v, v, (3, 7, 4))
    out = ops.embedding(idx.to(DEV), wt.to(DEV))
    assert out.shape == (n, 3, 7, 4, d)
    torch.testing.assert_close(out.cpu(), wt[:, idx])
    odd = torch.randn(2, 10, 3).to(dtype)          # row bytes not a multiple of 16
    i2 = torch.randint(0, 10, (6,))
    torch.testing.assert_close(ops.embedding(i2.to(DEV), odd.to(DEV)).cpu(), odd[:, i2])
    no_device_error()


def test_embedding_out_of_range_sets_error_word():
    wt = torch.randn(2, 10, 8, device=DEV)
    out = ops.embedding(torch.tensor([1, 10, 3], device=DEV), wt)
    assert _native.device_error() == 110
    assert float(out[:, 1].abs().sum()) == 0.0
    torch.testing.assert_close(out[:, 0], wt[:, 1])
    no_device_error()
