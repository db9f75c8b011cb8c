"""GPU behaviour of the CUDA-graph executor (compile=True): replays equal the
eager TracedWideModel (reference forward: wide_compiler/core/traced_wide.py:
450-532), a replay launches nothing through the library's launch path, and
a new input buffer or new parameter storage records a new graph."""
import pytest
import torch
import torch.nn as nn

import wide_compiler as wc
from wide_compiler import _native
from gpu_util import assert_fp32_close, assert_lowp_close, no_device_error

pytestmark = pytest.mark.gpu
DEV = 'cuda'


class _MLP(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(64, 128)
        self.fc2 = nn.Linear(128, 64)

    def forward(self, x):
        return self.fc2(torch.relu(self.fc1(x)))


class _Block(nn.Module):
    def __init__(self, c=64):
        super().__init__()
        self.c1 = nn.Conv2d(c, c, 3, padding=1)
        self.b1 = nn.BatchNorm2d(c)
        self.c2 = nn.Conv2d(c, c, 3, padding=1)
        self.b2 = nn.BatchNorm2d(c)

    def forward(self, x):
        return self.b2(self.c2(torch.relu(self.b1(self.c1(x))))) + x


def test_graphed_mlp_matches_eager_and_replays():
    torch.manual_seed(1)
    n, b = 12, 32
    models = [_MLP() for _ in range(n)]
    eager = wc.compile(models, torch.randn(b, 64)).to(DEV)
    graphed = wc.compile(models, torch.randn(b, 64), compile_model=True).to(DEV)
    x = torch.randn(b, n * 64, device=DEV)
    y0 = graphed(x)                      # records, then replays
    assert_fp32_close(y0, eager(x))
    torch.cuda.synchronize()
    host_before, before = _native.lib().widek_launch_count(), _native.launch_count()
    x.copy_(torch.randn(b, n * 64, device=DEV))
    y1 = graphed(x)                      # replay: same static output, new values
    torch.cuda.synchronize()
    assert _native.lib().widek_launch_count() == host_before     # no launch from the host
    rec = next(iter(graphed._graphs.values()))
    assert rec.launches >= 1 and _native.launch_count() == before + rec.launches   # the graph's kernels counted
    assert y1.data_ptr() == y0.data_ptr()
    assert_fp32_close(y1, eager(x))
    x2 = torch.randn(b, n * 64, device=DEV)   # another buffer: a second graph
    y2 = graphed(x2)
    assert y2.data_ptr() != y1.data_ptr() and len(graphed._graphs) == 2
    assert_fp32_close(y2, eager(x2))
    no_device_error()


def test_graphed_rerecords_after_dtype_change():
    torch.manual_seed(2)
    n, b = 4, 8
    models = [_MLP() for _ in range(n)]
    graphed = wc.compile(models, torch.randn(b, 64), compile_model=True).to(DEV)
    x = torch.randn(b, n * 64, device=DEV)
    graphed(x)
    graphed.to(torch.bfloat16)            # new parameter storage
    xb = x.to(torch.bfloat16)
    y = graphed(xb)
    ref = wc.compile(models, torch.randn(b, 64)).to(DEV, torch.bfloat16)(xb)
    assert y.dtype == torch.bfloat16
    assert_lowp_close(y, ref.double())
    no_device_error()


def test_graphed_resblock_bf16():
    torch.manual_seed(3)
    n, b, c, hw = 3, 2, 64, 16
    blocks = [_Block(c) for _ in range(n)]
    for blk in blocks:
        for bn in (blk.b1, blk.b2):
            bn.running_mean.normal_(0, 0.1)
            bn.running_var.uniform_(0.5, 1.5)
    eager = wc.compile(blocks, torch.randn(1, c, hw, hw)).to(DEV, torch.bfloat16).eval()
    graphed = wc.compile(blocks, torch.randn(1, c, hw, hw), compile_model=True).to(DEV, torch.bfloat16).eval()
    x = torch.randn(b, n * c, hw, hw, device=DEV).to(torch.bfloat16)
    for _ in range(2):
        y = graphed(x)
    assert_lowp_close(y, eager(x).double())
    no_device_error()


def test_large_inputs_run_eagerly():
    torch.manual_seed(4)
    models = [_MLP() for _ in range(2)]
    graphed = wc.compile(models, torch.randn(4, 64), compile_model=True).to(DEV)
    graphed.max_input_bytes = 1024
    x = torch.randn(8, 128, device=DEV)
    y = graphed(x)
    assert len(graphed._graphs) == 0
    assert_fp32_close(y, graphed._orig_mod(x))
    no_device_error()
