"""GPU parity: WideLinear (tcgen05 tensor-core kernel and the CUDA-core fp32
kernel), WideLayerNorm, elementwise glue and the pack/unpack kernels, each
against the golden fixtures (reference outputs) and the oracle."""
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


@pytest.mark.parametrize("name", golden_names('linear') + golden_names('layernorm'))
def test_golden_fp32(name):
    g = load_golden(name)
    mod = _build_from_state(g).to(DEV)
    y = mod(g['inputs']['x'].to(DEV))
    assert_fp32_close(y, g['outputs']['y'])


def _rand_linear(n, m, k, o, dtype, bias=True, seed=0):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(n, m, k, generator=gen).to(dtype)
    w = (torch.randn(n, o, k, generator=gen) / k ** 0.5).to(dtype)
    b = (torch.randn(n, o, generator=gen) * 0.1).to(dtype) if bias else None
    return x, w, b


@pytest.mark.parametrize("n,m,k,o", [
    (1, 128, 64, 256), (3, 1, 64, 64), (2, 127, 72, 200), (2, 129, 200, 264), (1, 300, 8, 8),
    (4, 256, 1024, 512), (2, 64, 128, 136), (5, 32, 64, 128), (1, 1000, 96, 40)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_tcgen05_shapes(n, m, k, o, dtype):
    x, w, b = _rand_linear(n, m, k, o, dtype, seed=n * 1000 + m + k + o)
    y = ops.linear(x.to(DEV), w.to(DEV), b.to(DEV))
    assert y.dtype == dtype and y.shape == (n, m, o)
    assert_lowp_close(y, O.linear(x, w, b))
    no_device_error()


@pytest.mark.parametrize("act,name", [(ops.ACT_RELU, 'relu'), (ops.ACT_GELU, 'gelu')])
def test_linear_epilogue_activation(act, name):
    x, w, b = _rand_linear(3, 200, 128, 192, torch.bfloat16, seed=7)
    y = ops.linear(x.to(DEV), w.to(DEV), b.to(DEV), act=act)
    assert_lowp_close(y, O.linear(x, w, b, act=name))
    y32 = ops.linear(x.float().to(DEV), w.float().to(DEV), b.float().to(DEV), act=act)
    assert_fp32_close(y32, O.linear(x.float(), w.float(), b.float(), act=name))


def test_linear_no_bias_and_batch_dims():
    x, w, _ = _rand_linear(2, 24, 64, 96, torch.bfloat16, bias=False, seed=3)
    x4 = x.view(2, 4, 6, 64)
    y = ops.linear(x4.to(DEV), w.to(DEV), None)
    assert y.shape == (2, 4, 6, 96)
    assert_lowp_close(y, O.linear(x4, w, None))


@pytest.mark.parametrize("n,m,k,o", [(100, 32, 64, 128), (100, 32, 128, 64), (3, 70, 33, 17), (1, 1, 1, 1)])
def test_linear_fp32_simt(n, m, k, o):
    x, w, b = _rand_linear(n, m, k, o, torch.float32, seed=m + k)
    y = ops.linear(x.to(DEV), w.to(DEV), b.to(DEV))
    assert_fp32_close(y, O.linear(x, w, b))


def test_linear_bf16_unaligned_k_uses_cuda_cores():
    x, w, b = _rand_linear(2, 50, 30, 40, torch.bfloat16, seed=9)   # k % 8 != 0
    y = ops.linear(x.to(DEV), w.to(DEV), b.to(DEV))
    assert_lowp_close(y, O.linear(x, w, b))


def test_linear_tc_matches_simt():
    x, w, b = _rand_linear(3, 256, 256, 384, torch.bfloat16, seed=11)
    xd, wd, bd = x.to(DEV), w.to(DEV), b.to(DEV)
    y_tc = ops.linear(xd, wd, bd)
    y_simt = ops.linear(xd, wd, bd, force_simt=True)
    assert_lowp_close(y_tc, y_simt.float(), rtol=1e-2)


def test_linear_cfg2_full_size_sampled():
    """Benchmark configuration cfg2 (N=64, 1024->4096, B=256, bf16) at full size; the oracle
    checks a sample of models and rows, a checksum covers every output."""
    n, m, k, o = 64, 256, 1024, 4096
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(n, m, k, device=DEV, generator=g, dtype=torch.float32).to(torch.bfloat16)
    w = (torch.randn(n, o, k, device=DEV, generator=g) / 32).to(torch.bfloat16)
    b = torch.zeros(n, o, device=DEV, dtype=torch.bfloat16)
    y = ops.linear(x, w, b)
    for i in (0, 17, 63):
        rows = torch.tensor([0, 1, 127, 128, 200, 255])
        ref = O.linear(x[i:i + 1, rows].cpu(), w[i:i + 1].cpu(), b[i:i + 1].cpu())
        assert_lowp_close(y[i:i + 1, rows], ref)
    # Every output: compare per-model column sums against an fp32 GEMM of the
    # same bf16 operands (sum over rows commutes with the contraction).
    ref_sum = torch.einsum('nk,nok->no', x.float().sum(1), w.float())
    torch.testing.assert_close(y.float().sum(1), ref_sum, rtol=2e-2, atol=0.5)
    no_device_error()


@pytest.mark.parametrize("d", [48, 512, 1000, 4096, 33])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_layernorm_shapes(d, dtype):
    n = 3
    g = torch.Generator().manual_seed(d)
    x = (torch.randn(n, 4, 7, d, generator=g) * 3 + 1).to(dtype)
    w = (torch.rand(n * d, generator=g) + 0.5).to(dtype)
    b = (torch.randn(n * d, generator=g) * 0.1).to(dtype)
    y = ops.layernorm(x.to(DEV), w.to(DEV), b.to(DEV), n, d, 1e-5)
    ref = O.layernorm(x, w, b, n, d, 1e-5)
    if dtype == torch.float32:
        assert_fp32_close(y, ref)
    else:
        assert_lowp_close(y, ref)


def test_layernorm_cfg5_full_size():
    n, d = 16, 512
    x = torch.randn(n, 8, 1024, d, device=DEV).to(torch.bfloat16)
    w = (torch.rand(n * d, device=DEV) + 0.5).to(torch.bfloat16)
    b = (torch.randn(n * d, device=DEV) * 0.1).to(torch.bfloat16)
    y = ops.layernorm(x, w, b, n, d, 1e-5)
    ref = O.layernorm(x.cpu(), w.cpu(), b.cpu(), n, d, 1e-5)
    assert_lowp_close(y, ref)


@pytest.mark.parametrize("op", ['relu', 'gelu', 'sigmoid', 'tanh', 'silu'])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_unary(op, dtype):
    x = (torch.randn(3, 5, 77) * 3).to(dtype)
    y = ops.unary(x.to(DEV), op)
    ref = O.activation(x.double(), op)
    (assert_fp32_close if dtype == torch.float32 else assert_lowp_close)(y, ref)


@pytest.mark.parametrize("op", ['add', 'mul', 'sub', 'div'])
def test_binary(op):
    a = torch.randn(4, 3, 33)
    b = torch.rand(4, 3, 33) + 0.5
    y = ops.binary(a.to(DEV), b.to(DEV), op)
    assert_fp32_close(y, O.binary(a, b, op))


@pytest.mark.parametrize("shape,dtype", [((3, 5, 7), torch.float32), ((4, 2, 64, 3, 3), torch.bfloat16),
                                         ((2, 3, 5), torch.bfloat16), ((100, 32, 64), torch.float32)])
def test_swap01_and_pack(shape, dtype):
    x = torch.randn(*shape).to(dtype)
    # byte-moving kernels: bit-exact
    y = ops.swap01(x.to(DEV))
    assert torch.equal(y.cpu(), x.transpose(0, 1).contiguous())
    inputs = [torch.randn(*shape[1:]).to(dtype) for _ in range(shape[0])]
    packed = wc.pack([t.to(DEV) for t in inputs])
    assert torch.equal(packed.cpu(), O.pack_inputs(inputs).to(dtype))
    outs = wc.unpack(packed, shape[0])
    for a, b in zip(outs, inputs):
        assert torch.equal(a.cpu(), b)


def test_pack_many_sources():
    inputs = [torch.randn(3, 8) for _ in range(150)]   # more than one launch of 64 pointers
    packed = wc.pack([t.to(DEV) for t in inputs])
    assert torch.equal(packed.cpu(), O.pack_inputs(inputs))


@pytest.mark.parametrize("shape", [(32, 6400, 32, 32), (7, 3, 5, 1, 9)])
def test_swap01_large_and_odd_bit_exact(shape):
    """The boundary transpose at cfg3's size (419 MB bf16) and at an odd
    shape whose rows are not 16-byte multiples."""
    g = torch.Generator(device=DEV).manual_seed(5)
    b, nc = shape[0], shape[1]
    x = torch.randn(*shape, device=DEV, generator=g).to(torch.bfloat16)
    n = 100 if nc == 6400 else 3
    xv = x.view(b, n, nc // n, *shape[2:])
    y = ops.swap01(xv)
    assert torch.equal(y, xv.transpose(0, 1).contiguous())
    assert torch.equal(ops.swap01(y), xv)


def test_traced_mlp_golden():
    g = load_golden('traced_mlp')
    n = g['meta']['n']
    import torch.nn as nn
    import torch.nn.functional as F

    class MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1 = nn.Linear(8, 16)
            self.fc2 = nn.Linear(16, 8)

        def forward(self, x):
            return self.fc2(F.relu(self.fc1(x)))

    models = []
    for i in range(n):
        m = MLP()
        m.load_state_dict({k.split('.', 1)[1]: v for k, v in g['state'].items() if k.startswith(f'm{i}.')})
        models.append(m.to(DEV).eval())
    wide = wc.compile(models, torch.randn(3, 8, device=DEV))
    out = wide(g['inputs']['packed'].to(DEV))
    assert_fp32_close(out, g['outputs']['y'])
    no_device_error()


@pytest.mark.parametrize("n,b,t,k,o,dtype", [
    (3, 4, 32, 64, 96, torch.bfloat16),      # T divides 128: box of 4 row blocks
    (2, 2, 256, 128, 64, torch.bfloat16),    # T a multiple of 128
    (4, 128, 1, 64, 200, torch.float16),     # T = 1 ([B, N*K] rows)
    (2, 3, 50, 64, 64, torch.bfloat16),      # T neither: CUDA-core kernel
    (2, 3, 16, 24, 40, torch.float32),       # fp32: CUDA-core kernel
])
@pytest.mark.parametrize("inp,outp", [(True, True), (True, False), (False, True)])
def test_linear_packed_rows(n, b, t, k, o, dtype, inp, outp):
    """widek_linear_fwd_ex on the packed boundary layout [B, N*T, K] (in,
    out or both) equals unpack -> linear -> pack, bit for bit against the
    N-first kernel call on the same inputs."""
    g = torch.Generator().manual_seed(n * 100 + t)
    x = torch.randn(n, b, t, k, generator=g).to(dtype)
    w = (torch.randn(n, o, k, generator=g) / k ** 0.5).to(dtype)
    bias = (torch.randn(n, o, generator=g) * 0.1).to(dtype)
    xd, wd, bd = x.to(DEV), w.to(DEV), bias.to(DEV)
    xin = O.nfirst_to_packed(x).reshape(b, n * t, k).contiguous().to(DEV) if inp else xd
    y = ops.linear_layout(xin, wd, bd, ops.ACT_NONE, inp, outp)
    ref = ops.linear(xd, wd, bd)
    if outp:
        ref = O.nfirst_to_packed(ref).reshape(b, n * t, o).to(DEV)
    assert y.shape == ref.shape
    if dtype == torch.float32 or t % 128 == 0 or 128 % t == 0:
        assert torch.equal(y, ref)          # same kernel, same tiles: bit-identical
    else:
        assert_lowp_close(y, ref.double())  # packed rows on the CUDA-core kernel
    if dtype == torch.float32:
        assert_fp32_close(ref if not outp else y, O.linear(x, w, bias) if not outp else
                          O.nfirst_to_packed(O.linear(x, w, bias)).reshape(b, n * t, o))
    no_device_error()


@pytest.mark.parametrize("n,m,k,o", [(2, 256, 1024, 512), (3, 300, 200, 264), (1, 129, 64, 136), (4, 512, 256, 1024),
                                     (2, 8192, 512, 1536)])
def test_linear_pair_tiles_match_single_cta(n, m, k, o):
    """CTA-pair (cta_group::2, 256x256 per pair) tiles against single-CTA
    tiles and the oracle: the same products in the same k order, so the
    results agree bit for bit."""
    from wide_compiler import _native
    x, w, b = _rand_linear(n, m, k, o, torch.bfloat16, seed=m + o)
    xd, wd, bd = x.to(DEV), w.to(DEV), b.to(DEV)
    lib = _native.lib()
    try:
        _native.check(lib.widek_linear_set_variant(1), "variant")
        y1 = ops.linear(xd, wd, bd)
        _native.check(lib.widek_linear_set_variant(2), "variant")
        y2 = ops.linear(xd, wd, bd)
        y2p = None
        if m % 32 == 0:
            # packed [B, n*T, k] rows (T = 32, B = m / 32): 4-D row-block maps
            xp = xd.view(n, m // 32, 32, k).transpose(0, 1).reshape(m // 32, n * 32, k).contiguous()
            y2p = ops.linear_layout(xp, wd, bd, ops.ACT_NONE, True, False)
    finally:
        lib.widek_linear_set_variant(0)
    assert torch.equal(y1, y2)
    if y2p is not None:
        assert torch.equal(y2p.reshape(y2.shape), y2)
    assert_lowp_close(y1[:, :64], O.linear(x[:, :64], w, b))
    no_device_error()


@pytest.mark.parametrize("n,m,k,o", [(3, 300, 100, 200), (2, 128, 64, 384), (4, 37, 256, 130), (1, 1000, 512, 64),
                                     (2, 64, 102, 96)])
def test_linear_fp32_split_tensor_core(n, m, k, o):
    """fp32 WideLinear on the split-operand tensor-core kernel (three bf16
    pieces, six products per K step) against the fp64 oracle at the fp32
    tolerance and against the CUDA-core kernel (linear variant 6); k = 102
    (not a multiple of 4) takes the CUDA-core kernel."""
    from wide_compiler import _native
    x, w, b = _rand_linear(n, m, k, o, torch.float32, seed=m + k)
    xd, wd, bd = x.to(DEV), w.to(DEV), b.to(DEV)
    lib = _native.lib()
    y = ops.linear(xd, wd, bd)
    try:
        _native.check(lib.widek_linear_set_variant(6), "variant")
        y_simt = ops.linear(xd, wd, bd)
    finally:
        lib.widek_linear_set_variant(0)
    ref = O.linear(x, w, b)
    assert_fp32_close(y, ref)
    assert_fp32_close(y_simt, ref)
    # the split products are as accurate as fp32 multiplies: the error
    # against fp64 is that of an fp32 GEMM (the CUDA-core kernel's), up to
    # accumulation order
    err = (y.double().cpu() - ref).abs().max().item()
    err_simt = (y_simt.double().cpu() - ref).abs().max().item()
    assert err <= 4 * max(err_simt, 1e-6 * ref.abs().max().item()), (err, err_simt)
    no_device_error()


def test_linear_fp32_split_unscaled_long_k():
    """Unscaled N(0, 1) operands and K = 2048 (sums of 2048 terms of order
    one, like a weight gradient summed over a large batch): the split kernel
    stays within the fp32 tolerance of fp64 and as close as the CUDA-core
    kernel."""
    from wide_compiler import _native
    g = torch.Generator().manual_seed(7)
    n, m, k, o = 2, 128, 2048, 128
    x = torch.randn(n, m, k, generator=g)
    w = torch.randn(n, o, k, generator=g)
    y = ops.linear(x.to(DEV), w.to(DEV), None)
    lib = _native.lib()
    try:
        _native.check(lib.widek_linear_set_variant(6), "variant")
        y_simt = ops.linear(x.to(DEV), w.to(DEV), None)
    finally:
        lib.widek_linear_set_variant(0)
    ref = O.linear(x, w, None)
    assert_fp32_close(y, ref)
    err = (y.double().cpu() - ref).abs().max().item()
    err_simt = (y_simt.double().cpu() - ref).abs().max().item()
    assert err <= 4 * err_simt + 1e-6, (err, err_simt)
    no_device_error()
