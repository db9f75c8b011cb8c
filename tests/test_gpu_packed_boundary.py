"""TracedWideModel graphs whose first / last stages are norms, elementwise
glue or recurrent layers run on the packed boundary layout [B, N*C, ...]
directly: no unpack / pack copy (ops.swap01) is launched, and the output
equals the per-model eager modules stacked by pack_inputs (the reference's
forward, wide_compiler/core/traced_wide.py:450-534, which unpacks at :463-469
and packs at :527-532). fp32 at rtol 1e-3 / atol 1e-4."""
import copy

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from wide_compiler import ops
from wide_compiler.core.traced_wide import TracedWideModel
from gpu_util import assert_fp32_close, assert_lowp_close, no_device_error
from oracle import wide_oracle as O

pytestmark = pytest.mark.gpu
DEV = 'cuda'


@pytest.fixture
def swap_calls(monkeypatch):
    calls = []
    real = ops.swap01

    def counting(x):
        calls.append(tuple(x.shape))
        return real(x)
    monkeypatch.setattr(ops, 'swap01', counting)
    return calls


def _run(models, sample, inputs):
    wide = TracedWideModel.from_models(models, sample).eval()
    out = wide(O.pack_inputs(inputs).to(DEV))
    with torch.no_grad():
        outs = [m(x) for m, x in zip(models, inputs)]
        ref = O.pack_inputs([o[0] if isinstance(o, tuple) else o for o in outs])
    return out, ref


class NormGlue(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.bn = nn.BatchNorm2d(c)
        self.gn = nn.GroupNorm(4, c)

    def forward(self, x):
        y = F.relu(self.bn(x))
        return self.gn(y) + x * 0.5


class LNGlue(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.ln = nn.LayerNorm(d)

    def forward(self, x):
        return torch.sigmoid(self.ln(x)) * x


class GRUHead(nn.Module):
    def __init__(self, i, h):
        super().__init__()
        self.gru = nn.GRU(i, h, batch_first=True)
        self.ln = nn.LayerNorm(h)

    def forward(self, x):
        out, _ = self.gru(x)
        return self.ln(out)


class LSTMOnly(nn.Module):
    def __init__(self, i, h):
        super().__init__()
        self.lstm = nn.LSTM(i, h, batch_first=True)

    def forward(self, x):
        out, _ = self.lstm(x)
        return out


class INorm(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.inorm = nn.InstanceNorm1d(c, affine=True)

    def forward(self, x):
        return F.gelu(self.inorm(x))


def _models(cls, n, *a):
    torch.manual_seed(7)
    ms = []
    for _ in range(n):
        m = cls(*a)
        with torch.no_grad():
            for name, b in m.named_buffers():
                if name.endswith('running_mean'):
                    b.uniform_(-0.5, 0.5)
                elif name.endswith('running_var'):
                    b.uniform_(0.5, 1.5)
            for p in m.parameters():
                if p.dim() == 1:
                    p.uniform_(0.5, 1.5)
        ms.append(m.to(DEV).eval())
    return ms


@pytest.mark.parametrize("case", ["bn_gn_glue", "ln_glue_3d", "ln_glue_2d", "gru_ln", "lstm", "instancenorm"])
def test_packed_boundary_graphs(case, swap_calls):
    n, b = 5, 3
    g = torch.Generator().manual_seed(3)
    if case == "bn_gn_glue":
        models, shape = _models(NormGlue, n, 16), (b, 16, 6, 7)
    elif case == "ln_glue_3d":
        models, shape = _models(LNGlue, n, 40), (b, 9, 40)
    elif case == "ln_glue_2d":
        models, shape = _models(LNGlue, n, 24), (b, 24)
    elif case == "gru_ln":
        models, shape = _models(GRUHead, n, 12, 32), (b, 10, 12)
    elif case == "lstm":
        models, shape = _models(LSTMOnly, n, 8, 24), (b, 7, 8)
    else:
        models, shape = _models(INorm, n, 12), (b, 12, 20)
    inputs = [torch.randn(*shape, generator=g).to(DEV) for _ in range(n)]
    with torch.no_grad():
        out, ref = _run(models, inputs[0], inputs)
    assert_fp32_close(out, ref)
    assert swap_calls == [], f"{case}: unpack/pack copies {swap_calls}"
    no_device_error()


def test_packed_training_batchnorm_updates_running_stats(swap_calls):
    """A training-mode BatchNorm first stage on the packed layout updates the
    running statistics exactly as the per-model modules do."""
    n, b = 4, 6
    models = _models(NormGlue, n, 8)
    for m in models:
        m.train()
    g = torch.Generator().manual_seed(4)
    inputs = [torch.randn(b, 8, 5, 5, generator=g).to(DEV) for _ in range(n)]
    wide = TracedWideModel.from_models(models, inputs[0]).train()
    with torch.no_grad():
        out = wide(O.pack_inputs(inputs).to(DEV))
        ref = O.pack_inputs([m(x) for m, x in zip(models, inputs)])
    assert_fp32_close(out, ref)
    bn = wide.stages['bn'].op
    assert_fp32_close(bn.running_mean, torch.cat([m.bn.running_mean for m in models]))
    assert_fp32_close(bn.running_var, torch.cat([m.bn.running_var for m in models]))
    assert swap_calls == []
    no_device_error()


def test_unpacked_consumer_still_gets_one_unpack(swap_calls):
    """A stage without a packed form (here a transpose of the last two
    dims) after a packed LayerNorm gets the N-first tensor through one
    unpack, and the output is packed once at the end."""
    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.ln = nn.LayerNorm(16)

        def forward(self, x):
            return self.ln(x).transpose(-1, -2)

    n, b = 3, 4
    models = _models(M, n)
    g = torch.Generator().manual_seed(5)
    inputs = [torch.randn(b, 6, 16, generator=g).to(DEV) for _ in range(n)]
    with torch.no_grad():
        out, ref = _run(models, inputs[0], inputs)
    assert_fp32_close(out, ref)
    assert len(swap_calls) == 2      # unpack before the matmul, pack at the end
    no_device_error()


class MHALN(nn.Module):
    def __init__(self, d, h):
        super().__init__()
        self.attn = nn.MultiheadAttention(d, h, batch_first=True)
        self.ln = nn.LayerNorm(d)

    def forward(self, x):
        a, _ = self.attn(x, x, x, need_weights=False)
        return self.ln(a + x)


class Seq3D(nn.Module):
    def __init__(self, k, h, o):
        super().__init__()
        self.fc1 = nn.Linear(k, h)
        self.fc2 = nn.Linear(h, o)

    def forward(self, x):
        return self.fc2(F.gelu(self.fc1(x)))


@pytest.mark.parametrize("case", ["mha_ln", "linear_3d", "gru_ln_bf16"])
def test_packed_boundary_matches_unfused_bitwise(case, swap_calls):
    """bf16 attention / Linear / GRU graphs: the packed-layout run launches
    no unpack / pack copy and gives bit-identical results to the N-first
    run (fuse=False: unpack, the same kernels, pack), which in turn matches
    the per-model modules at the bf16 tolerance."""
    n, b = 4, 3
    torch.manual_seed(11)
    if case == "mha_ln":
        models = [MHALN(128, 2) for _ in range(n)]
        shape = (b, 64, 128)
    elif case == "linear_3d":
        models = [Seq3D(64, 128, 32) for _ in range(n)]
        shape = (b, 32, 64)
    else:
        models = [GRUHead(64, 64) for _ in range(n)]
        shape = (b, 16, 64)
    models = [m.to(DEV, torch.bfloat16).eval() for m in models]
    g = torch.Generator().manual_seed(12)
    inputs = [torch.randn(*shape, generator=g).to(DEV, torch.bfloat16) for _ in range(n)]
    packed = O.pack_inputs(inputs).to(DEV)
    with torch.no_grad():
        wide = TracedWideModel.from_models(models, inputs[0]).eval()
        fused = wide(packed)
        assert swap_calls == [], f"{case}: unpack/pack copies {swap_calls}"
        if case == "linear_3d":
            # the N-first run of the same fused layers (GELU in fc1's epilogue)
            st = wide.stages
            h = ops.linear(O.packed_to_nfirst(packed.cpu(), n).to(DEV), st['fc1'].weight, st['fc1'].bias,
                           act=ops.ACT_GELU)
            plain = O.nfirst_to_packed(ops.linear(h, st['fc2'].weight, st['fc2'].bias)).reshape(fused.shape)
            plain = plain.to(DEV)
        else:
            wide.fuse = False
            wide._fusion = None
            plain = wide(packed)
            assert len(swap_calls) == 2
        # fp32 copies of the same (bf16-rounded) modules on the same inputs
        ref = O.pack_inputs([copy.deepcopy(m).float()(x.float()) for m, x in zip(models, inputs)])
    assert torch.equal(fused, plain)
    assert_lowp_close(fused, ref)
    no_device_error()
