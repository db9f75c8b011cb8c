"""Test configuration: import paths, the ``gpu`` marker, fixture helpers.

* ``-m "not gpu"`` tests run on any machine: the oracle against the golden
  fixtures, host-side logic, and the C-ABI library's exports.
* ``-m gpu`` tests need a B200: they call the CUDA kernels (through the
  primitives or the C-ABI directly) and compare with the oracle / fixtures.
"""
from __future__ import annotations

import glob
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "pytorch-parallel-compiler_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; runs the sm_100a kernels")
    config.addinivalue_line("markers", "grad: runs with autograd enabled (gradient tests)")


def golden_names(kind=None):
    names = sorted(os.path.basename(p)[:-3] for p in glob.glob(os.path.join(GOLDEN, "*.pt")))
    if kind is None:
        return names
    return [n for n in names if load_golden(n)["kind"] == kind]


_cache = {}


def load_golden(name):
    if name not in _cache:
        _cache[name] = torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=False)
    return _cache[name]


def cuda_ok() -> bool:
    return torch.cuda.is_available()


@pytest.fixture(autouse=True)
def _no_tf32():
    # fp32 parity is defined with TF32 off (reference tolerance contract).
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield


@pytest.fixture(autouse=True)
def _inference_unless_grad(request):
    # Forward-parity GPU tests run as inference (the fused kernels and the
    # graph executor serve calls whose result autograd does not need); tests
    # marked ``grad`` exercise the differentiable path.
    if request.node.get_closest_marker("gpu") and not request.node.get_closest_marker("grad"):
        with torch.no_grad():
            yield
    else:
        yield
