"""Failure detection on the GPU without a fault: a kernel whose bounded wait
cannot be satisfied (an mbarrier nothing arrives at) must give up after its
limit, report the timeout through the device error word that the host reads
(widek_device_error), and leave the context usable for the next launch.
The reference has no device code; its failures are Python exceptions
(wide_compiler/core/registry.py:48-51, api.py:105-122), which the C-ABI's
status codes mirror."""
import time

import pytest
import torch

from wide_compiler import _native as N
from wide_compiler import ops
from gpu_util import assert_fp32_close
from oracle import wide_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


def test_bounded_wait_runs_out_and_reports():
    lib = N.load()
    assert N.device_error() == 0
    t0 = time.perf_counter()
    N.check(lib.widek_test_bounded_wait(2_000_000, N.stream_ptr(DEV)), "widek_test_bounded_wait")  # 2 ms
    code = N.device_error()                  # synchronizes
    elapsed = time.perf_counter() - t0
    assert code == N.DEV_ERR_WAIT_PROBE
    assert elapsed < 5.0, f"the bounded wait took {elapsed:.2f} s"
    assert N.device_error() == 0             # read-and-clear
    # the context is still usable: a kernel launches and computes correctly
    x = torch.randn(2, 5, 16, device=DEV)
    w = torch.randn(2, 8, 16, device=DEV)
    b = torch.randn(2, 8, device=DEV)
    assert_fp32_close(ops.linear(x, w, b), O.linear(x.cpu(), w.cpu(), b.cpu()))
    assert N.device_error() == 0


def test_timeout_code_maps_to_an_exception_at_the_boundary():
    """The host turns a non-zero error word into an exception for callers
    that ask for it (the pattern the primitives' tests use)."""
    lib = N.load()
    N.check(lib.widek_test_bounded_wait(1_000_000, N.stream_ptr(DEV)), "widek_test_bounded_wait")
    with pytest.raises(AssertionError):
        assert N.device_error() == 0
    assert N.device_error() == 0
