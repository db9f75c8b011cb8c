"""GPU parity of the one-launch Linear chain (widek_mlp_chain_fwd): a run of
WideLinear layers with activations, N-first or packed in and out, against the
float64 oracle of the reference's per-layer path (WideLinear einsum + bias,
wide_compiler/core/primitives/wide_linear.py:165-168, the activation node,
and the TracedWideModel boundary unpack/pack, core/traced_wide.py:450-532).
"""
import pytest
import torch
import torch.nn as nn

import wide_compiler as wc
from wide_compiler import _native, ops
from gpu_util import assert_fp32_close, assert_lowp_close, kernels_run, no_device_error
from oracle import wide_oracle as O

pytestmark = pytest.mark.gpu
DEV = 'cuda'
ACT_NAMES = {ops.ACT_NONE: 'none', ops.ACT_RELU: 'relu', ops.ACT_GELU: 'gelu'}


def _chain(n, dims, dtype, bias=True, seed=0):
    gen = torch.Generator().manual_seed(seed)
    ws, bs = [], []
    for din, dout in zip(dims[:-1], dims[1:]):
        ws.append((torch.randn(n, dout, din, generator=gen) / din ** 0.5).to(dtype))
        bs.append((torch.randn(n, dout, generator=gen) * 0.1).to(dtype) if bias else None)
    return ws, bs


def _oracle(x_nfirst, ws, bs, acts, dtype):
    """Layer by layer in float64, each layer's output rounded to the storage
    dtype as a per-layer run stores it."""
    h = x_nfirst
    for w, b, a in zip(ws, bs, acts):
        h = O.linear(h, w, b, act=ACT_NAMES[a]).to(dtype)
    return h


def _check(y, ref, dtype):
    if dtype == torch.float32:
        assert_fp32_close(y, ref)
    else:
        assert_lowp_close(y, ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("in_l,out_l", [(0, 0), (1, 1), (1, 0), (0, 1)])
def test_cfg1_shape_layouts(dtype, in_l, out_l):
    """The benchmark cfg1 MLP (64 -> 128, ReLU, -> 64), every layout pair."""
    n, b, dims, acts = 7, 32, [64, 128, 64], [ops.ACT_RELU, ops.ACT_NONE]
    ws, bs = _chain(n, dims, dtype, seed=1)
    x = torch.randn(n, b, dims[0], generator=torch.Generator().manual_seed(2)).to(dtype)
    xin = O.nfirst_to_packed(x).contiguous() if in_l == 1 else x
    y = ops.mlp_chain(xin.to(DEV), [w.to(DEV) for w in ws], [t.to(DEV) for t in bs], acts, n, in_l, out_l)
    assert y is not None
    ref = _oracle(x, ws, bs, acts, dtype)
    if out_l == 1:
        assert y.shape == (b, n * dims[-1])
        ref = O.nfirst_to_packed(ref)
    else:
        assert y.shape == (n, b, dims[-1])
    _check(y, ref, dtype)
    no_device_error()


@pytest.mark.parametrize("n,b,dims,acts", [
    (3, 5, [5, 7, 3], [ops.ACT_GELU, ops.ACT_RELU]),             # ragged widths and batch
    (2, 1, [33, 65, 129, 17], [ops.ACT_RELU, ops.ACT_GELU, ops.ACT_NONE]),
    (1, 37, [64, 64], [ops.ACT_NONE]),                            # one layer, rows split across CTAs
    (4, 9, [16] * 9, [ops.ACT_RELU] * 8),                         # eight layers
    (2, 300, [200, 200, 200], [ops.ACT_RELU, ops.ACT_NONE]),      # weights loaded one layer at a time
    (2, 2000, [128, 96, 128], [ops.ACT_GELU, ops.ACT_RELU]),      # batch split to fit shared memory
])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_chain_shapes(n, b, dims, acts, dtype):
    ws, bs = _chain(n, dims, dtype, seed=n + b + len(dims))
    x = torch.randn(n, b, dims[0], generator=torch.Generator().manual_seed(b)).to(dtype)
    y = ops.mlp_chain(x.to(DEV), [w.to(DEV) for w in ws], [t.to(DEV) for t in bs], acts, n)
    assert y is not None and y.shape == (n, b, dims[-1])
    _check(y, _oracle(x, ws, bs, acts, dtype), dtype)
    no_device_error()


def test_chain_without_bias_f16():
    n, b, dims, acts = 5, 16, [48, 80, 24], [ops.ACT_RELU, ops.ACT_NONE]
    ws, bs = _chain(n, dims, torch.float16, bias=False, seed=5)
    x = torch.randn(n, b, dims[0], generator=torch.Generator().manual_seed(6)).to(torch.float16)
    y = ops.mlp_chain(x.to(DEV), [w.to(DEV) for w in ws], bs, acts, n)
    _check(y, _oracle(x, ws, bs, acts, torch.float16), torch.float16)
    no_device_error()


def test_chain_too_large_is_declined():
    """A chain whose one layer of weights exceeds shared memory returns None
    and launches nothing; the widths are still checked."""
    n, dims = 1, [512, 512]
    ws, bs = _chain(n, dims, torch.float32)
    before = _native.launch_count()
    assert ops.mlp_chain(torch.randn(n, 4, 512, device=DEV), [ws[0].to(DEV)], [bs[0].to(DEV)], [0], n) is None
    assert _native.launch_count() == before
    with pytest.raises(ValueError):
        ops.mlp_chain(torch.randn(n, 4, 100, device=DEV), [ws[0].to(DEV)], [bs[0].to(DEV)], [0], n)


def test_zero_batch_is_noop():
    ws, bs = _chain(2, [8, 8], torch.float32)
    y = ops.mlp_chain(torch.empty(2, 0, 8, device=DEV), [ws[0].to(DEV)], [bs[0].to(DEV)], [0], 2)
    assert y is not None and y.shape == (2, 0, 8)


class _MLP(nn.Module):
    def __init__(self, i=64, h=128, o=64):
        super().__init__()
        self.fc1 = nn.Linear(i, h)
        self.fc2 = nn.Linear(h, o)

    def forward(self, x):
        return self.fc2(torch.relu(self.fc1(x)))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_traced_mlp_one_launch(dtype):
    """The compiled N-MLP ensemble (packed in, packed out) runs as exactly one
    library launch and equals the node-by-node run of the same model."""
    torch.manual_seed(3)
    n, b = 10, 32
    model = wc.compile([_MLP() for _ in range(n)], torch.randn(b, 64)).to(DEV, dtype)
    x = torch.randn(b, n * 64, device=DEV).to(dtype)
    model(x)
    torch.cuda.synchronize()
    before = _native.launch_count()
    y = model(x)
    torch.cuda.synchronize()
    assert _native.launch_count() - before == 1
    model.fuse = False
    model._fusion = None
    y_plain = model(x)
    assert y.shape == y_plain.shape == (b, n * 64)
    _check(y, y_plain.double(), dtype)
    no_device_error()


def test_traced_mlp_matches_per_model_modules():
    """Against the N template modules run one by one in float64 (the
    reference's N x nn.Module baseline), for a deeper chain with GELU."""
    class Deep(nn.Module):
        def __init__(self):
            super().__init__()
            self.a = nn.Linear(20, 40)
            self.b = nn.Linear(40, 40)
            self.c = nn.Linear(40, 12)

        def forward(self, x):
            return self.c(torch.relu(self.b(nn.functional.gelu(self.a(x)))))

    torch.manual_seed(9)
    n, b = 6, 11
    models = [Deep() for _ in range(n)]
    wide = wc.compile(models, torch.randn(b, 20)).to(DEV)
    xs = [torch.randn(b, 20) for _ in range(n)]
    y = wide(wc.pack_inputs([xi.to(DEV) for xi in xs]))
    outs = wc.unpack_outputs(y, n)
    for m, xi, yi in zip(models, xs, outs):
        assert_fp32_close(yi, m.double()(xi.double()))
    no_device_error()


@pytest.mark.parametrize("n,b,dims,acts,bias,fits", [
    (7, 32, [64, 128, 64], [ops.ACT_RELU, ops.ACT_NONE], True, True),             # cfg1 shape
    (5, 16, [32, 64, 32, 8], [ops.ACT_GELU, ops.ACT_RELU, ops.ACT_NONE], True, True),  # 3 layers, narrow
    (3, 40, [20, 128, 12], [ops.ACT_RELU, ops.ACT_NONE], False, True),       # ragged widths (K padding), no bias
    (2, 64, [64, 64, 64], [ops.ACT_GELU, ops.ACT_GELU], True, True),         # activation on the last layer
    (3, 300, [64, 128, 96, 32], [ops.ACT_GELU, ops.ACT_RELU, ops.ACT_NONE], True, False),   # too large: CUDA cores
    (2, 8, [36, 128, 128, 128, 12], [ops.ACT_RELU] * 3 + [ops.ACT_NONE], True, False),
])
@pytest.mark.parametrize("in_l,out_l", [(0, 0), (1, 1), (0, 1)])
def test_fp32_chain_tensor_core_vs_cuda_cores(n, b, dims, acts, bias, fits, in_l, out_l):
    """fp32 chains on the tcgen05 split-operand kernel (chain variant 1,
    where its plan fits in shared memory; checked by kernel name) and on the
    CUDA-core kernel (variant 0, the default), both against the fp64 oracle
    at the fp32 tolerance."""
    ws, bs = _chain(n, dims, torch.float32, bias=bias, seed=b + len(dims))
    x = torch.randn(n, b, dims[0], generator=torch.Generator().manual_seed(b)).to(torch.float32)
    xin = (O.nfirst_to_packed(x).contiguous() if in_l == 1 else x).to(DEV)
    wd = [w.to(DEV) for w in ws]
    bd = [t.to(DEV) if t is not None else None for t in bs]
    ref = _oracle(x, ws, bs, acts, torch.float32)
    if out_l == 1:
        ref = O.nfirst_to_packed(ref)
    lib = _native.lib()
    got = {}
    try:
        _native.check(lib.widek_mlp_chain_set_variant(1), "variant")     # tensor cores wherever they fit
        names = kernels_run(lambda: got.__setitem__('tc', ops.mlp_chain(xin, wd, bd, acts, n, in_l, out_l)))
        _native.check(lib.widek_mlp_chain_set_variant(0), "variant")
        got['cc'] = ops.mlp_chain(xin, wd, bd, acts, n, in_l, out_l)
    finally:
        lib.widek_mlp_chain_set_variant(0)
    assert got['tc'] is not None and got['cc'] is not None
    assert any('mlp_chain_tc_kernel' in k for k in names) == fits, names
    assert_fp32_close(got['tc'], ref)
    assert_fp32_close(got['cc'], ref)
    no_device_error()
