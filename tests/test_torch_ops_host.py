"""Host-side checks of the torch.library operators (namespace ``widek``) that
let dynamo / torch.compile trace the wide primitives (the reference's quick
start compiles WideGRU with torch.compile, reference README.md:65): every
operator is registered, and each fake implementation gives the shapes,
dtypes and devices of the op's torch formulation (the reference's
arithmetic) without running a kernel. Runs without a GPU (fake CUDA
tensors)."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import wide_compiler  # noqa: F401  (registers the operators)
from wide_compiler import _autograd as AG
from wide_compiler import _torch_ops


def test_every_operator_is_registered():
    for name in _torch_ops.OPERATORS:
        assert hasattr(torch.ops.widek, name), name


def _same(a, b):
    a = a if isinstance(a, tuple) else (a,)
    b = b if isinstance(b, tuple) else (b,)
    assert len(a) == len(b)
    for x, y in zip(a, b):
        assert tuple(x.shape) == tuple(y.shape) and x.dtype == y.dtype and x.device == y.device, (x, y)


def test_fake_implementations_match_the_torch_formulations():
    with FakeTensorMode():
        dev = 'cuda'
        t = lambda *s, dt=torch.float32: torch.empty(*s, device=dev, dtype=dt)
        n, b = 3, 2
        x = t(n, b, 5, 16)
        w, bias = t(n, 24, 16), t(n, 24)
        _same(torch.ops.widek.linear(x, w, bias, 1), AG.linear_t(x, w, bias, 1))
        lw, lb = t(n * 16), t(n * 16)
        _same(torch.ops.widek.layernorm(x, lw, lb, n, 16, 1e-5), AG.layernorm_t(x, lw, lb, n, 16, 1e-5))
        xc = t(n, b, 8, 6, 6, dt=torch.bfloat16)
        cw, cb = t(n * 8, dt=torch.bfloat16), t(n * 8, dt=torch.bfloat16)
        _same(torch.ops.widek.batchnorm(xc, n, 8, cw, cb, t(n * 8, dt=torch.bfloat16), t(n * 8, dt=torch.bfloat16),
                                        True, True, 0.1, 1e-5),
              AG.batchnorm_t(xc, n, 8, cw, cb, None, None, True, False, 0.1, 1e-5))
        _same(torch.ops.widek.groupnorm(xc, n, 4, cw, cb, 1e-5), AG.groupnorm_t(xc, n, 4, cw, cb, 1e-5))
        idx = torch.empty(4, 7, device=dev, dtype=torch.int64)
        ew = t(n, 50, 12)
        _same(torch.ops.widek.embedding(idx, ew), AG.embedding_t(idx, ew))
        kw = t(n * 10, 8, 3, 3, dt=torch.bfloat16)
        _same(torch.ops.widek.conv(xc, kw, None, n, [2, 1], [1, 0], [1, 2]),
              AG.conv_nd_t(xc, kw, None, n, (2, 1), (1, 0), (1, 2)))
        wih, whh, bih, bhh = t(n, 3 * 32, 16), t(n, 3 * 32, 32), t(n, 96), t(n, 96)
        _same(torch.ops.widek.gru(x, None, wih, whh, bih, bhh), AG.gru_t(x, None, wih, whh, bih, bhh))
        bd_ih, bd_hh = t(n * 128, n * 16), t(n * 128, n * 32)
        _same(torch.ops.widek.lstm(x, None, None, bd_ih, bd_hh, t(n, 128), t(n, 128), n, 32),
              _torch_ops._lstm_blockdiag_t(x, None, None, bd_ih, bd_hh, t(n, 128), t(n, 128), n, 32))
        q = t(n, b, 9, 32, dt=torch.bfloat16)
        qw, kvw, ow = t(n, 32, 32, dt=torch.bfloat16), t(n, 64, 32, dt=torch.bfloat16), t(n, 32, 32, dt=torch.bfloat16)
        _same(torch.ops.widek.attention(q, q, q, qw, None, kvw, None, ow, None, 4, None, True, True),
              AG.attention_t(q, q, q, None, True, 4, qw, None, kvw, None, ow, None))
        _same(torch.ops.widek.swap01(x), AG.swap01_t(x))
        _same(torch.ops.widek.unary(x, 'gelu'), AG.unary_t(x, 'gelu'))
        _same(torch.ops.widek.binary(x, x, 'mul'), AG.binary_t(x, x, 'mul'))
