"""GPU parity: WideAttention (projection GEMMs + flash attention core)
against the reference fixtures and the oracle."""
import pytest
import torch

import wide_compiler as wc
from wide_compiler import ops
from conftest import golden_names, load_golden
from gpu_util import assert_fp32_close, assert_lowp_close, kernels_run as _kernels_run, no_device_error
from oracle import wide_oracle as O
from test_api_host import _build_from_state

pytestmark = pytest.mark.gpu
DEV = 'cuda'


@pytest.mark.parametrize("name", golden_names('attention'))
def test_attention_golden(name):
    g = load_golden(name)
    mod = _build_from_state(g).to(DEV).eval()
    inp = g['inputs']
    q = inp['q'].to(DEV)
    k = inp['k'].to(DEV) if inp['k'] is not None else None
    v = inp['v'].to(DEV) if inp['v'] is not None else None
    mask = inp['mask'].to(DEV) if inp['mask'] is not None else None
    out = mod(q, k, v, attn_mask=mask, is_causal=g['meta']['causal'])
    if g['meta']['tuple']:
        assert isinstance(out, tuple) and out[1] is None
        out = out[0]
    assert_fp32_close(out, g['outputs']['y'])


def _mod(n, d, h, dtype, seed):
    torch.manual_seed(seed)
    m = wc.WideAttention(n, d, h)
    with torch.no_grad():
        m.q_bias.normal_(0, 0.1)
        m.kv_bias.normal_(0, 0.1)
        m.out_bias.normal_(0, 0.1)
    return m.to(DEV, dtype).eval()


def _ref(m, q, k, v, mask=None, causal=False):
    p = {k_: (v_.detach().cpu() if v_ is not None else None) for k_, v_ in m.named_parameters()}
    return O.attention(q.cpu(), k.cpu(), v.cpu(), p['q_weight'], p['kv_weight'], p['q_bias'], p['kv_bias'],
                       p['out_weight'], p['out_bias'], m.n_heads, None if mask is None else mask.cpu(), causal)


@pytest.mark.parametrize("n,b,t,d,h", [(2, 3, 100, 256, 4), (3, 2, 64, 512, 8), (2, 2, 130, 256, 2), (1, 1, 1, 128, 2)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_bf16_self(n, b, t, d, h, causal):
    m = _mod(n, d, h, torch.bfloat16, n + t)
    x = torch.randn(n, b, t, d, device=DEV).to(torch.bfloat16)
    y = m(x, is_causal=causal)
    assert_lowp_close(y, _ref(m, x, x, x, causal=causal))
    no_device_error()


def test_attention_bf16_cross_and_separate_value():
    m = _mod(2, 128, 2, torch.bfloat16, 3)
    q = torch.randn(2, 3, 70, 128, device=DEV).to(torch.bfloat16)
    kv = torch.randn(2, 3, 45, 128, device=DEV).to(torch.bfloat16)
    v = torch.randn(2, 3, 45, 128, device=DEV).to(torch.bfloat16)
    out, none = m(q, kv, kv)
    assert none is None
    assert_lowp_close(out, _ref(m, q, kv, kv))
    out2, _ = m(q, kv, v)
    assert_lowp_close(out2, _ref(m, q, kv, v))


@pytest.mark.parametrize("kind", ['bool', 'float', 'float32', 'per_head'])
def test_attention_masks_bf16(kind):
    n, b, t, d, h = 2, 2, 80, 256, 4
    m = _mod(n, d, h, torch.bfloat16, 11)
    x = torch.randn(n, b, t, d, device=DEV).to(torch.bfloat16)
    if kind == 'bool':
        mask = torch.rand(t, t, device=DEV) > 0.4
        mask[:, 0] = True
    elif kind == 'float':
        mask = torch.randn(t, t, device=DEV).to(torch.bfloat16)
    elif kind == 'float32':
        mask = torch.randn(t, t, device=DEV)
    else:
        mask = torch.randn(n * b, h, t, t, device=DEV).to(torch.bfloat16)
    y = m(x, attn_mask=mask)
    assert_lowp_close(y, _ref(m, x, x, x, mask=mask))


def test_attention_fp32_modules_match_torch_mha():
    torch.manual_seed(0)
    mhas = [torch.nn.MultiheadAttention(64, 4, batch_first=True).eval() for _ in range(3)]
    w = wc.WideAttention.from_modules(mhas).to(DEV).eval()
    x = torch.randn(3, 2, 20, 64)
    out, _ = w(x.to(DEV), x.to(DEV), x.to(DEV), is_causal=False)
    for i in range(3):
        ref, _ = mhas[i](x[i], x[i], x[i], need_weights=False)
        assert_fp32_close(out[i], ref.detach())


def test_attention_cfg5_full_size_sampled():
    """Benchmark configuration cfg5: N=16, B=8, T=1024, d=512, 8 heads, causal, bf16; the
    oracle checks two (model, batch) slices."""
    n, b, t, d, h = 16, 8, 1024, 512, 8
    torch.manual_seed(5)
    m = wc.WideAttention(n, d, h)
    with torch.no_grad():
        for p in (m.q_weight, m.kv_weight, m.out_weight):
            p.normal_(0, 0.02)
        m.q_bias.zero_(); m.kv_bias.zero_(); m.out_bias.zero_()
    m = m.to(DEV, torch.bfloat16).eval()
    x = torch.randn(n, b, t, d, device=DEV).to(torch.bfloat16)
    y = m(x, is_causal=True)
    for i, j in ((0, 0), (15, 7)):
        sub = wc.WideAttention(1, d, h).to(DEV, torch.bfloat16)
        with torch.no_grad():
            for name, p in sub.named_parameters():
                p.copy_(getattr(m, name)[i:i + 1])
        xs = x[i:i + 1, j:j + 1]
        ref = _ref(sub, xs, xs, xs, causal=True)
        assert_lowp_close(y[i:i + 1, j:j + 1], ref)
    no_device_error()


@pytest.mark.parametrize("kind", ['bool', 'float', 'float32', 'per_head'])
@pytest.mark.parametrize("t,causal", [(80, False), (75, False), (200, True)])
def test_attention_masks_on_tcgen05(kind, t, causal):
    """Explicit masks (wide_attention.py:223-228) run on the tcgen05 flash
    kernel: bool (attend where true) and additive (bf16 or fp32) masks,
    broadcast [T, T] or per (sample, head), vectorised (T a multiple of the
    16-byte vector) and scalar (T = 75) mask reads, alone and with the causal
    mask; rows whose keys are all masked give zeros, as the other kernels."""
    n, b, d, h = 2, 2, 256, 4
    m = _mod(n, d, h, torch.bfloat16, 21 + t)
    x = torch.randn(n, b, t, d, device=DEV).to(torch.bfloat16)
    g = torch.Generator(device=DEV).manual_seed(t)
    if kind == 'bool':
        mask = torch.rand(t, t, device=DEV, generator=g) > 0.4
        mask[:, 0] = True
        mask[3, :] = False                   # one query attends nothing
    elif kind == 'float':
        mask = torch.randn(t, t, device=DEV, generator=g).to(torch.bfloat16)
    elif kind == 'float32':
        mask = torch.randn(t, t, device=DEV, generator=g)
    else:
        mask = torch.randn(n * b, h, t, t, device=DEV, generator=g).to(torch.bfloat16)
    names = _kernels_run(lambda: m(x, attn_mask=mask, is_causal=False) if not causal else None)
    if not causal:
        assert any('attn_tc_kernel' in s for s in names), names
    y = m(x, attn_mask=mask) if not causal else None
    if causal:
        # is_causal with an explicit mask is rejected (SDPA's rule); the
        # causal + mask combination is the mask with the upper triangle off
        tri = torch.ones(t, t, device=DEV, dtype=torch.bool).tril()
        cm = (mask & tri) if kind == 'bool' else mask.float().masked_fill(~tri, float('-inf')).to(mask.dtype)
        y = m(x, attn_mask=cm)
        ref = _ref(m, x, x, x, mask=cm)
    else:
        ref = _ref(m, x, x, x, mask=mask)
    # a query with no attended key: zeros from the core (the oracle's
    # softmax over only -inf gives NaN), so the module returns out_bias
    nan_rows = torch.isnan(ref).any(dim=-1)
    ref = torch.where(nan_rows[..., None], m.out_bias.detach().double().cpu()[:, None, None, :], ref)
    assert_lowp_close(y, ref)
    if kind == 'bool' and not causal:
        assert torch.count_nonzero(y[:, :, 3].float() - m.out_bias[:, None, :].float()) == 0
    no_device_error()
