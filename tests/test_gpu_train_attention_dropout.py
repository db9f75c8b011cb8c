"""WideAttention in training mode with attention dropout (reference
wide_attention.py:221-228: SDPA with dropout_p = module dropout while
training). The projections run on the WideLinear kernels and their backward
kernels; the core is torch's SDPA with dropout. Checked against the
reference's formulation (einsum projections, SDPA with dropout) run on the
same GPU from the same seed, so that both draw the same mask: forward and
every parameter gradient within the fp32 contract (rtol 1e-3 / atol 1e-4).
"""
import math

import pytest
import torch
import torch.nn.functional as F

import wide_compiler as wc
from gpu_util import assert_fp32_close, no_device_error

pytestmark = [pytest.mark.gpu, pytest.mark.grad]
DEV = torch.device('cuda', 0)


def _reference(params, n, d, heads, dropout, x, is_causal):
    qw, qb, kvw, kvb, ow, ob = params
    _, b, t, _ = x.shape
    dh = d // heads
    q = torch.einsum('nbtd,nod->nbto', x, qw) + qb.view(n, 1, 1, d)
    k = torch.einsum('nbtd,nod->nbto', x, kvw[:, :d]) + kvb[:, :d].view(n, 1, 1, d)
    v = torch.einsum('nbtd,nod->nbto', x, kvw[:, d:]) + kvb[:, d:].view(n, 1, 1, d)
    # the same head views as the module's path, so SDPA picks the same
    # backend and draws the same dropout mask from the same seed
    split = lambda u: u.reshape(n * b, t, heads, dh).transpose(1, 2)
    o = F.scaled_dot_product_attention(split(q), split(k), split(v), dropout_p=dropout, is_causal=is_causal,
                                       scale=1.0 / math.sqrt(dh))
    o = o.transpose(1, 2).reshape(n, b, t, d)
    return torch.einsum('nbtd,nod->nbto', o, ow) + ob.view(n, 1, 1, d)


@pytest.mark.parametrize("is_causal", [False, True])
def test_attention_dropout_training_matches_reference(is_causal):
    torch.manual_seed(3)
    n, d, heads, p = 2, 64, 2, 0.2
    mod = wc.WideAttention(n, d, heads, dropout=p).to(DEV).train()
    with torch.no_grad():
        for b in (mod.q_bias, mod.kv_bias, mod.out_bias):
            b.normal_(0, 0.1)
    x = torch.randn(n, 3, 16, d, device=DEV)
    names = ('q_weight', 'q_bias', 'kv_weight', 'kv_bias', 'out_weight', 'out_bias')
    dy = torch.randn(n, 3, 16, d, device=DEV)

    torch.manual_seed(7)
    got = mod(x, is_causal=is_causal)
    got.backward(dy)
    torch.cuda.synchronize()
    no_device_error()

    ref_params = [getattr(mod, k).detach().clone().requires_grad_(True) for k in names]
    torch.manual_seed(7)
    want = _reference(ref_params, n, d, heads, p, x, is_causal)
    want.backward(dy)

    assert_fp32_close(got.detach(), want.detach())
    for k, r in zip(names, ref_params):
        assert_fp32_close(getattr(mod, k).grad, r.grad)
    # the mask is random: another seed gives another output
    torch.manual_seed(8)
    with torch.no_grad():
        assert not torch.allclose(mod(x, is_causal=is_causal), got.detach())
