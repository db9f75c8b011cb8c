"""GPU parity: WideGRU / WideLSTM persistent recurrence kernels against the
reference fixtures and the oracle (fp32 contract: rtol 1e-3 / atol 1e-4)."""
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


@pytest.mark.parametrize("name", golden_names('gru') + golden_names('lstm'))
def test_rnn_golden(name):
    g = load_golden(name)
    mod = _build_from_state(g).to(DEV)
    inp = g['inputs']
    x = inp['x'].to(DEV)
    if g['kind'] == 'gru':
        h0 = inp['h0'].to(DEV) if inp['h0'] is not None else None
        y, hn = mod(x, h0)
        assert_fp32_close(y, g['outputs']['y'])
        assert_fp32_close(hn, g['outputs']['h_n'])
    else:
        hx = (inp['h0'].to(DEV), inp['c0'].to(DEV)) if inp['h0'] is not None else None
        y, (hn, cn) = mod(x, hx)
        assert_fp32_close(y, g['outputs']['y'])
        assert_fp32_close(hn, g['outputs']['h_n'])
        assert_fp32_close(cn, g['outputs']['c_n'])


def _rnn_params(n, i, h, gates, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    s = 1.0 / h ** 0.5
    u = lambda *shape: ((torch.rand(*shape, generator=gen) * 2 - 1) * s).to(dtype)
    return u(n, gates * h, i), u(n, gates * h, h), u(n, gates * h), u(n, gates * h)


@pytest.mark.parametrize("n,b,t,i,h", [(32, 4, 32, 64, 128), (3, 16, 7, 20, 256), (2, 3, 5, 8, 24), (1, 1, 1, 4, 8)])
def test_gru_random_fp32(n, b, t, i, h):
    wih, whh, bih, bhh = _rnn_params(n, i, h, 3, torch.float32, n + h)
    x = torch.randn(n, b, t, i)
    h0 = torch.randn(n, b, h) * 0.5
    y, hn = ops.gru(x.to(DEV), h0.to(DEV), wih.to(DEV), whh.to(DEV), bih.to(DEV), bhh.to(DEV))
    ry, rh = O.gru(x, h0, wih, whh, bih, bhh)
    assert_fp32_close(y, ry)
    assert_fp32_close(hn, rh)
    no_device_error()


@pytest.mark.parametrize("n,b,t,i,h", [(32, 4, 32, 64, 128), (2, 8, 6, 16, 512), (3, 5, 4, 12, 40), (2, 40, 3, 8, 64)])
def test_lstm_random_fp32(n, b, t, i, h):
    wih, whh, bih, bhh = _rnn_params(n, i, h, 4, torch.float32, n * 7 + h)
    x = torch.randn(n, b, t, i)
    h0, c0 = torch.randn(n, b, h) * 0.5, torch.randn(n, b, h) * 0.5
    y, (hn, cn) = ops.lstm(x.to(DEV), h0.to(DEV), c0.to(DEV), wih.to(DEV), whh.to(DEV), bih.to(DEV), bhh.to(DEV))
    ry, (rh, rc) = O.lstm(x, h0, c0, wih, whh, bih, bhh)
    assert_fp32_close(y, ry)
    assert_fp32_close(hn, rh)
    assert_fp32_close(cn, rc)
    no_device_error()


def test_rnn_bf16_and_no_bias():
    n, b, t, i, h = 4, 4, 16, 32, 128
    wih, whh, _, _ = _rnn_params(n, i, h, 3, torch.bfloat16, 5)
    x = torch.randn(n, b, t, i).to(torch.bfloat16)
    y, hn = ops.gru(x.to(DEV), None, wih.to(DEV), whh.to(DEV), None, None)
    ry, rh = O.gru(x, None, wih, whh, None, None)
    assert_lowp_close(y, ry)
    wih, whh, bih, bhh = _rnn_params(n, i, h, 4, torch.bfloat16, 6)
    y, (hn, cn) = ops.lstm(x.to(DEV), None, None, wih.to(DEV), whh.to(DEV), bih.to(DEV), bhh.to(DEV))
    ry, (rh, rc) = O.lstm(x, None, None, wih, whh, bih, bhh)
    assert_lowp_close(y, ry)
    assert_lowp_close(cn, rc)


def test_rnn_modules_from_torch_cfg4():
    """Benchmark configuration cfg4 through the public modules built from nn.GRU / nn.LSTM."""
    torch.manual_seed(0)
    grus = [torch.nn.GRU(64, 128, batch_first=True) for _ in range(32)]
    lstms = [torch.nn.LSTM(64, 128, batch_first=True) for _ in range(32)]
    x = torch.randn(32, 4, 32, 64)
    wg = wc.WideGRU.from_modules(grus).to(DEV)
    wl = wc.WideLSTM.from_modules(lstms).to(DEV)
    y, hn = wg(x.to(DEV))
    for k in (0, 13, 31):
        ry, rh = grus[k](x[k])
        assert_fp32_close(y[k], ry.detach())
        assert_fp32_close(hn[k], rh[0].detach())
    y, (hn, cn) = wl(x.to(DEV))
    for k in (0, 31):
        ry, (rh, rc) = lstms[k](x[k])
        assert_fp32_close(y[k], ry.detach())
        assert_fp32_close(cn[k], rc[0].detach())


def test_rnn_zero_steps():
    wih, whh, bih, bhh = _rnn_params(2, 4, 8, 3, torch.float32, 1)
    h0 = torch.randn(2, 3, 8)
    y, hn = ops.gru(torch.empty(2, 3, 0, 4, device=DEV), h0.to(DEV), wih.to(DEV), whh.to(DEV), bih.to(DEV),
                    bhh.to(DEV))
    assert y.shape == (2, 3, 0, 8)
    torch.testing.assert_close(hn.cpu(), h0)


@pytest.fixture(params=[0, 1], ids=["register-resident", "smem-cluster"])
def rnn_variant(request):
    from wide_compiler import _native as N
    N.check(N.lib().widek_rnn_set_variant(request.param), "widek_rnn_set_variant")
    yield request.param
    N.lib().widek_rnn_set_variant(0)


@pytest.mark.parametrize("n,b,t", [(32, 4, 32), (1, 1, 5), (5, 8, 9), (2, 40, 3), (100, 2, 4)])
@pytest.mark.parametrize("kind", ["gru", "lstm"])
def test_rnn_h128_both_kernels(rnn_variant, kind, n, b, t):
    """Hidden size 128, where the register-resident kernel applies (cluster
    sizes 8/4/2 by N; N=100 leaves one CTA per model and takes the
    shared-memory kernel); batch 40 makes the gate loop stride; both kernels
    against the oracle."""
    i, h = 24, 128
    g = 3 if kind == "gru" else 4
    wih, whh, bih, bhh = _rnn_params(n, i, h, g, torch.float32, n * 11 + b + t + g)
    x = torch.randn(n, b, t, i, generator=torch.Generator().manual_seed(b + t))
    h0 = torch.randn(n, b, h, generator=torch.Generator().manual_seed(n)) * 0.5
    if kind == "gru":
        y, hn = ops.gru(x.to(DEV), h0.to(DEV), wih.to(DEV), whh.to(DEV), bih.to(DEV), bhh.to(DEV))
        ry, rh = O.gru(x, h0, wih, whh, bih, bhh)
    else:
        c0 = torch.randn(n, b, h, generator=torch.Generator().manual_seed(n + 1)) * 0.5
        y, (hn, cn) = ops.lstm(x.to(DEV), h0.to(DEV), c0.to(DEV), wih.to(DEV), whh.to(DEV), bih.to(DEV),
                               bhh.to(DEV))
        ry, (rh, rc) = O.lstm(x, h0, c0, wih, whh, bih, bhh)
        assert_fp32_close(cn, rc)
    assert_fp32_close(y, ry)
    assert_fp32_close(hn, rh)
    no_device_error()


# ---------------------------------------------------------------------------
# One-call GRU / LSTM forward (projection with strided W_ih, then the
# recurrence with strided W_hh): WideLSTM passes its block-diagonal
# parameters as they are
# ---------------------------------------------------------------------------

def _blockdiag(blocks):
    """[N, R, C] dense blocks -> the [N*R, N*C] block-diagonal module layout."""
    n, r, c = blocks.shape
    out = torch.zeros(n * r, n * c, dtype=blocks.dtype)
    for k in range(n):
        out[k * r:(k + 1) * r, k * c:(k + 1) * c] = blocks[k]
    return out


@pytest.mark.parametrize("n,b,t,i,h,bias,dtype", [
    (32, 4, 32, 64, 128, True, torch.float32),     # cfg4
    (5, 3, 9, 20, 128, True, torch.float32),
    (2, 1, 1, 4, 128, False, torch.float32),
    (7, 17, 6, 128, 128, True, torch.float32),
    (3, 5, 4, 12, 40, True, torch.float32),        # shared-memory cluster kernel
    (4, 4, 16, 32, 128, True, torch.bfloat16),
])
def test_blockdiag_lstm_and_gru_match_oracle(n, b, t, i, h, bias, dtype):
    close = assert_fp32_close if dtype == torch.float32 else assert_lowp_close
    gen = torch.Generator().manual_seed(n * 13 + b + t + i)
    x = torch.randn(n, b, t, i, generator=gen).to(dtype)
    h0 = (torch.randn(n, b, h, generator=gen) * 0.5).to(dtype)
    c0 = (torch.randn(n, b, h, generator=gen) * 0.5).to(dtype)
    dv = lambda v: None if v is None else v.to(DEV)
    wih, whh, bih, bhh = _rnn_params(n, i, h, 3, dtype, n + i)
    if not bias:
        bih = bhh = None
    y, hn = ops.gru(x.to(DEV), h0.to(DEV), wih.to(DEV), whh.to(DEV), dv(bih), dv(bhh))
    ry, rh = O.gru(x, h0, wih, whh, bih, bhh)
    close(y, ry)
    close(hn, rh)
    wih, whh, bih, bhh = _rnn_params(n, i, h, 4, dtype, n + i + 1)
    if not bias:
        bih = bhh = None
    y, (hn, cn) = ops.lstm_blockdiag(x.to(DEV), h0.to(DEV), c0.to(DEV), _blockdiag(wih).to(DEV),
                                     _blockdiag(whh).to(DEV), dv(bih), dv(bhh), n, h)
    ry, (rh, rc) = O.lstm(x, h0, c0, wih, whh, bih, bhh)
    close(y, ry)
    close(hn, rh)
    close(cn, rc)
    no_device_error()


def test_one_call_matches_projection_then_recurrence():
    """widek_gru_fwd against the two separate entry points (grouped GEMM for
    the projection, then widek_gru_recurrence) on the same inputs."""
    from wide_compiler import _native as N
    n, b, t, i, h = 6, 5, 12, 48, 128
    wih, whh, bih, bhh = (v.to(DEV) for v in _rnn_params(n, i, h, 3, torch.float32, 77))
    x = torch.randn(n, b, t, i, generator=torch.Generator().manual_seed(3)).to(DEV)
    y1, h1 = ops.gru(x, None, wih, whh, bih, bhh)
    gx = ops.linear(x, wih, bih)
    y2 = torch.empty_like(y1)
    h2 = torch.empty_like(h1)
    N.check(N.lib().widek_gru_recurrence(gx.data_ptr(), whh.data_ptr(), bhh.data_ptr(), None, y2.data_ptr(),
                                         h2.data_ptr(), n, b, t, h, N.F32, N.stream_ptr(x.device)),
            "widek_gru_recurrence")
    assert_fp32_close(y1, y2)
    assert_fp32_close(h1, h2)
    no_device_error()


def test_wide_lstm_module_reads_block_diagonal_in_place():
    """WideLSTM's forward reads its block-diagonal parameters in place (no
    extracted blocks are cached) and follows an in-place update."""
    torch.manual_seed(5)
    lstms = [torch.nn.LSTM(16, 128, batch_first=True) for _ in range(3)]
    wl = wc.WideLSTM.from_modules(lstms).to(DEV)
    x = torch.randn(3, 2, 7, 16, device=DEV)
    y, _ = wl(x)
    assert not getattr(wl, '_widek_derived', None), "no derived blocks on the inference path"
    ry, _ = lstms[1](x[1].cpu())
    assert_fp32_close(y[1], ry.detach())
    with torch.no_grad():
        wl.weight_hh.mul_(0.5)
        for m in lstms:
            m.weight_hh_l0.mul_(0.5)
    y, (hn, cn) = wl(x)
    ry, (rh, rc) = lstms[2](x[2].cpu())
    assert_fp32_close(y[2], ry.detach())
    assert_fp32_close(cn[2], rc[0].detach())
    y0, (h0n, c0n) = wl(torch.empty(3, 2, 0, 16, device=DEV))
    assert y0.shape == (3, 2, 0, 128) and float(h0n.abs().max()) == 0.0
    no_device_error()
