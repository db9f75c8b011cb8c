"""torch.compile over the wide primitives (the reference's quick start,
README.md:65: ``torch.compile(WideGRU.from_modules(grus),
mode='reduce-overhead')``; its compile() does the same for a
TracedWideModel, wide_compiler/api.py:137-147). Dynamo traces the primitives
through the torch.library operators widek::* (no graph break inside a
primitive), the compiled module matches eager and the oracle, and gradients
flow through the operators' autograd formulas."""
import pytest
import torch
import torch.nn as nn

import wide_compiler as wc
from gpu_util import assert_fp32_close, assert_lowp_close, no_device_error
from oracle import wide_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


def _reset():
    torch._dynamo.reset()


def test_compiled_wide_gru_reduce_overhead_matches_eager():
    _reset()
    torch.manual_seed(0)
    grus = [nn.GRU(64, 128, batch_first=True) for _ in range(8)]
    wide = wc.WideGRU.from_modules(grus).to(DEV)
    x = torch.randn(8, 4, 16, 64, device=DEV)
    explanation = torch._dynamo.explain(wide)(x)
    assert explanation.graph_break_count == 0, explanation.break_reasons
    compiled = torch.compile(wide, mode='reduce-overhead')
    with torch.no_grad():
        for _ in range(3):                            # warm-up, record, replay
            y, hn = compiled(x)
        y, hn = y.clone(), hn.clone()
        ry, rh = wide(x)
    assert_fp32_close(y, ry)
    assert_fp32_close(hn, rh)
    for k in (0, 7):
        oy, oh = grus[k](x[k].cpu())
        assert_fp32_close(y[k], oy.detach())
    no_device_error()


def test_compiled_traced_model_matches_eager():
    """TracedWideModel (MLP with GELU and a residual) under torch.compile."""
    _reset()

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1 = nn.Linear(32, 64)
            self.fc2 = nn.Linear(64, 32)
            self.ln = nn.LayerNorm(32)

        def forward(self, x):
            return self.ln(self.fc2(torch.nn.functional.gelu(self.fc1(x))) + x)

    torch.manual_seed(1)
    models = [Block() for _ in range(5)]
    wide = wc.compile(models, torch.randn(4, 32)).to(DEV)
    x = torch.randn(4, 5 * 32, device=DEV)
    explanation = torch._dynamo.explain(wide)(x)
    assert explanation.graph_break_count == 0, explanation.break_reasons
    compiled = torch.compile(wide)
    with torch.no_grad():
        y = compiled(x)
        ref = wide(x)
    assert_fp32_close(y, ref)
    xs = wc.unpack(x, 5)
    expect = torch.cat([models[i].to(DEV)(xs[i]) for i in range(5)], dim=1)
    assert_fp32_close(y, expect.detach())
    no_device_error()


def test_compiled_attention_and_conv_bf16():
    _reset()
    torch.manual_seed(2)
    attn = wc.WideAttention(4, 128, 2).to(DEV, torch.bfloat16).eval()
    ln = wc.WideLayerNorm(4, 128).to(DEV, torch.bfloat16)
    convs = [nn.Conv2d(64, 64, 3, padding=1) for _ in range(3)]
    wconv = wc.WideConv2d.from_modules(convs).to(DEV, torch.bfloat16)
    x = torch.randn(4, 2, 64, 128, device=DEV).to(torch.bfloat16)
    xc = torch.randn(3, 2, 64, 16, 16, device=DEV).to(torch.bfloat16)
    f = lambda a, c: (ln(attn(a, is_causal=True)), wconv(c))
    explanation = torch._dynamo.explain(f)(x, xc)
    assert explanation.graph_break_count == 0, explanation.break_reasons
    compiled = torch.compile(f)
    with torch.no_grad():
        y, yc = compiled(x, xc)
        ry, ryc = f(x, xc)
    assert_lowp_close(y, ry.double())
    assert_lowp_close(yc, ryc.double())
    no_device_error()


@pytest.mark.grad
def test_compiled_training_step_gradients():
    """Gradients through the operators' autograd formulas under torch.compile
    equal the eager ones."""
    _reset()
    torch.manual_seed(3)
    lin = wc.WideLinear(3, 16, 24).to(DEV)
    x = torch.randn(3, 5, 16, device=DEV, requires_grad=True)
    compiled = torch.compile(lambda t: torch.nn.functional.gelu(lin(t)).square().sum())
    loss = compiled(x)
    loss.backward()
    gx, gw = x.grad.clone(), lin.weight.grad.clone()
    x.grad = None
    lin.weight.grad = None
    ref = torch.nn.functional.gelu(torch.einsum('noi,nbi->nbo', lin.weight, x) + lin.bias.unsqueeze(1))
    ref.square().sum().backward()
    assert_fp32_close(gx, x.grad)
    assert_fp32_close(gw, lin.weight.grad)
    no_device_error()
