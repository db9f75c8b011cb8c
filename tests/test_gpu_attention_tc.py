"""GPU parity of the attention core alone (widek_attention_fwd) on the
tcgen05/TMEM kernel (bf16/f16, head_dim 64, no explicit mask) and on the
warp-level MMA kernel (variant 1), against a float64 restatement of
scaled_dot_product_attention (the call the reference makes at
wide_compiler/core/primitives/wide_attention.py:217-231).

q/k/v are read through row strides from one fused [nb, t, 3*heads*64]
buffer, as the module's fused projection lays them out."""
import math

import pytest
import torch

from wide_compiler import _native as N
from wide_compiler import ops
from gpu_util import assert_lowp_close, no_device_error

pytestmark = pytest.mark.gpu
DEV = 'cuda'
DH = 64


def _sdpa64(q, k, v, causal):
    """q: [nb, heads, tq, dh], k/v: [nb, heads, tk, dh] -> float64 output."""
    q, k, v = q.double().cpu(), k.double().cpu(), v.double().cpu()
    s = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
    if causal:
        tq, tk = s.shape[-2:]
        keep = torch.ones(tq, tk, dtype=torch.bool).tril()
        s = s.masked_fill(~keep, float('-inf'))
    return torch.softmax(s, dim=-1) @ v


def _run(nb, heads, tq, tk, causal, dtype, variant, q_scale=1.0, key_ramp=0.0, seed=0):
    torch.manual_seed(seed)
    w = heads * DH
    qkv_q = torch.randn(nb, tq, 3 * w, device=DEV)
    qkv_k = qkv_q if tq == tk else torch.randn(nb, tk, 3 * w, device=DEV)
    qkv_q[..., :w] *= q_scale
    if key_ramp:
        ramp = 1.0 + key_ramp * torch.arange(tk, device=DEV, dtype=torch.float32) / max(tk, 1)
        qkv_k[..., w:2 * w] *= ramp.view(1, tk, 1)
    qkv_q = qkv_q.to(dtype)
    qkv_k = qkv_k.to(dtype) if qkv_k is not qkv_q else qkv_q
    q = qkv_q[..., :w]
    k = qkv_k[..., w:2 * w]
    v = qkv_k[..., 2 * w:]
    out = torch.empty(nb, tq, w, device=DEV, dtype=dtype)
    N.check(N.lib().widek_attention_set_variant(variant), "widek_attention_set_variant")
    try:
        ops.attention_core(q, k, v, nb, heads, tq, tk, DH, 3 * w, 3 * w, 3 * w, out, causal, None)
        torch.cuda.synchronize()
    finally:
        N.lib().widek_attention_set_variant(0)
    sp = lambda u, t: u.float().view(nb, t, heads, DH).permute(0, 2, 1, 3)
    ref = _sdpa64(sp(q, tq), sp(k, tk), sp(v, tk), causal)
    ref = ref.permute(0, 2, 1, 3).reshape(nb, tq, w)
    return out, ref


SHAPES = [
    (2, 2, 256, 256),     # one CTA per head, both query tiles full
    (1, 3, 300, 300),     # second CTA: 44 rows in tile 0, tile 1 empty
    (2, 1, 1000, 1000),   # last CTA: tile 1 partly filled
    (1, 2, 128, 77),      # fewer keys than queries, ragged key tile
    (1, 2, 77, 300),      # more keys than queries
    (1, 1, 1, 1),
    (1, 2, 513, 129),     # ragged on both sides, one key past a tile
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("variant", [0, 1, 10, 12])
def test_core_bf16(shape, causal, variant):
    """variant 0: tcgen05 kernel (default exponential split), 1: warp-level
    MMA kernel, 10 / 12: tcgen05 with 0 / 2 of every 4 exponential pairs on
    the FMA-pipe polynomial."""
    nb, heads, tq, tk = shape
    out, ref = _run(nb, heads, tq, tk, causal, torch.bfloat16, variant, seed=tq + tk)
    assert_lowp_close(out, ref)
    no_device_error()


@pytest.mark.parametrize("causal", [False, True])
def test_core_f16(causal):
    out, ref = _run(2, 2, 384, 384, causal, torch.float16, 0, seed=7)
    assert_lowp_close(out, ref)
    no_device_error()


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("variant", [0, 12])
def test_core_large_scores_rescale(causal, variant):
    """Score spread of several units of log2 per tile and key norms growing
    along the sequence: the running max moves by more than 2^8 between tiles,
    so the output is rescaled in TMEM during the key loop."""
    out, ref = _run(2, 2, 640, 640, causal, torch.bfloat16, variant, q_scale=6.0, key_ramp=3.0, seed=11)
    assert_lowp_close(out, ref)
    no_device_error()


def test_core_variants_agree_cfg5_shape():
    """cfg5's core (T=1024, 8 heads, causal) on a few (model, batch) rows:
    the tcgen05 and warp-MMA kernels agree with each other and the float64
    restatement."""
    out0, ref = _run(4, 8, 1024, 1024, True, torch.bfloat16, 0, seed=5)
    out1, _ = _run(4, 8, 1024, 1024, True, torch.bfloat16, 1, seed=5)
    assert_lowp_close(out0, ref)
    assert_lowp_close(out1, ref)
    assert (out0.float() - out1.float()).abs().max().item() < 0.05
    no_device_error()


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("variant", [0, 10])
def test_core_persistent_rounds(causal, variant):
    """At least as many heads as SMs: one CTA per SM loops over work items
    (query blocks of 256 rows, heaviest first per round); 160 heads leave the
    last round partly empty and T=600 gives three query blocks, the last one
    ragged, so items of different sizes follow each other on a CTA."""
    out, ref = _run(20, 8, 600, 600, causal, torch.bfloat16, variant, seed=21)
    assert_lowp_close(out, ref)
    no_device_error()


def test_core_persistent_cross_lengths():
    """Persistent mode with tq != tk (keys past the causal diagonal)."""
    out, ref = _run(19, 8, 300, 520, True, torch.bfloat16, 0, seed=22)
    assert_lowp_close(out, ref)
    no_device_error()


def test_core_large_head_count_grid():
    """More than 65535 (batch x head) pairs: the tcgen05 kernel's flat grid."""
    nb, heads, t = 8200, 8, 8
    out, ref = _run(nb, heads, t, t, True, torch.bfloat16, 0, seed=3)
    assert_lowp_close(out, ref)
    no_device_error()


def test_exp2_polynomial_error_bound():
    """The FMA-pipe exponential (variant 12 puts half of the pairs on it):
    uniform scores make every probability equal, so the output is the exact
    mean of v up to the bf16 rounding of P; compare both exponential paths on
    a case whose scores span the polynomial's whole reduced range."""
    nb, heads, t = 1, 2, 512
    torch.manual_seed(1)
    w = heads * DH
    qkv = torch.randn(1, t, 3 * w, device=DEV)
    qkv[..., :w] *= 3.0
    qkv = qkv.to(torch.bfloat16)
    outs = []
    for variant in (10, 12):
        out = torch.empty(nb, t, w, device=DEV, dtype=torch.bfloat16)
        N.check(N.lib().widek_attention_set_variant(variant), "widek_attention_set_variant")
        try:
            ops.attention_core(qkv[..., :w], qkv[..., w:2 * w], qkv[..., 2 * w:], nb, heads, t, t, DH, 3 * w, 3 * w,
                               3 * w, out, False, None)
            torch.cuda.synchronize()
        finally:
            N.lib().widek_attention_set_variant(0)
        outs.append(out.float())
    # ex2.approx and the polynomial differ by < 1e-4 relative per entry, far
    # below the bf16 rounding of P (2^-9): outputs agree to bf16 precision.
    diff = (outs[0] - outs[1]).abs().max().item()
    assert diff <= 2e-2 * outs[0].abs().max().item(), diff
    no_device_error()
