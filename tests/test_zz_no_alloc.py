"""The allocation-free BatchNorm-train entry point, called through the C-ABI.

widek_batchnorm_train_fwd_noalloc serves callers that cannot allocate device
memory (a runtime that owns all device memory in its own fixed pool, a
latency-critical path that must not risk cudaMalloc's implicit device
synchronization, an FFI binding with no allocator). It keeps its scratch in
a fixed array inside the library instead of a caller workspace. This test
checks, on two calls in a row, that its outputs and running-statistics
updates match the workspace entry point (widek_batchnorm_train_fwd) within
the tolerances the other GPU tests use, and that oversize requests are
refused. It lives in its own file, collected last, and passes both alone in
a fresh process and after the rest of the suite.
"""
import ctypes

import pytest
import torch

from wide_compiler import _native as N
from gpu_util import assert_fp32_close, assert_lowp_close

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def _workspace_call(lib, x, w, b, rm, rv, n, bsz, c, l, dt):
    ws_bytes = lib.widek_batchnorm_train_workspace(n, bsz, c, l)
    ws = torch.empty(max(int(ws_bytes), 16), dtype=torch.uint8, device=DEV)
    y = torch.empty_like(x)
    rc = lib.widek_batchnorm_train_fwd(x.data_ptr(), y.data_ptr(), w.data_ptr(), b.data_ptr(), rm.data_ptr(),
                                       rv.data_ptr(), None, None, ws.data_ptr(), ws.numel(), n, bsz, c, l, 0.1, 1e-5,
                                       dt, torch.cuda.current_stream().cuda_stream)
    N.check(rc, "widek_batchnorm_train_fwd")
    return y


def _noalloc_call(lib, x, w, b, rm, rv, n, bsz, c, l, dt, save_mean=None, save_invstd=None):
    y = torch.empty_like(x)
    rc = lib.widek_batchnorm_train_fwd_noalloc(
        x.data_ptr(), y.data_ptr(), w.data_ptr(), b.data_ptr(), rm.data_ptr(), rv.data_ptr(),
        None if save_mean is None else ctypes.cast(save_mean.data_ptr(), ctypes.POINTER(ctypes.c_float)),
        None if save_invstd is None else ctypes.cast(save_invstd.data_ptr(), ctypes.POINTER(ctypes.c_float)),
        n, bsz, c, l, 0.1, 1e-5, dt, torch.cuda.current_stream().cuda_stream)
    N.check(rc, "widek_batchnorm_train_fwd_noalloc")
    return y


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_workspace_entry_point_two_calls(dtype):
    lib = N.load()
    dt = N.dtype_code(torch.empty(0, dtype=dtype))
    close = assert_fp32_close if dtype == torch.float32 else assert_lowp_close
    g = torch.Generator(device=DEV).manual_seed(0)
    n, bsz, c, h, w_ = 8, 16, 64, 16, 16
    l = h * w_
    wt = (torch.rand(n * c, device=DEV, generator=g) + 0.5).to(dtype)
    bs = (torch.randn(n * c, device=DEV, generator=g) * 0.1).to(dtype)
    rm_ref = torch.randn(n * c, device=DEV, generator=g).to(dtype)
    rv_ref = (torch.rand(n * c, device=DEV, generator=g) + 0.5).to(dtype)
    rm_new, rv_new = rm_ref.clone(), rv_ref.clone()
    for call in range(2):
        x = (torch.randn(n, bsz, c, h, w_, device=DEV, generator=g) * (1.5 + call) + call).to(dtype)
        y_ref = _workspace_call(lib, x, wt, bs, rm_ref, rv_ref, n, bsz, c, l, dt)
        y_new = _noalloc_call(lib, x, wt, bs, rm_new, rv_new, n, bsz, c, l, dt)
        torch.cuda.synchronize()
        close(y_new, y_ref.double())
        close(rm_new, rm_ref.double())
        close(rv_new, rv_ref.double())
    assert N.device_error() == 0


def test_noalloc_saved_statistics_and_many_chunks():
    """Few channels with many elements, so the reduction is split into many
    chunks per channel (their partial sums all live in the fixed array);
    saved mean / inverse std match the batch statistics."""
    lib = N.load()
    n, bsz, c, l = 2, 64, 3, 4096
    x = torch.randn(n, bsz, c, l, device=DEV) * 2 + 1
    wt = torch.ones(n * c, device=DEV)
    bs = torch.zeros(n * c, device=DEV)
    rm = torch.zeros(n * c, device=DEV)
    rv = torch.ones(n * c, device=DEV)
    sm = torch.empty(n * c, device=DEV)
    si = torch.empty(n * c, device=DEV)
    for _ in range(2):
        y = _noalloc_call(lib, x, wt, bs, rm, rv, n, bsz, c, l, N.F32, sm, si)
    xr = x.double().permute(0, 2, 1, 3).reshape(n * c, -1)
    assert_fp32_close(sm, xr.mean(1))
    assert_fp32_close(si, 1.0 / torch.sqrt(xr.var(1, unbiased=False) + 1e-5))
    ref = (xr - xr.mean(1, keepdim=True)) / torch.sqrt(xr.var(1, unbiased=False, keepdim=True) + 1e-5)
    assert_fp32_close(y.double().permute(0, 2, 1, 3).reshape(n * c, -1), ref)


def test_noalloc_rejects_more_channels_than_the_fixed_scratch():
    lib = N.load()
    x = torch.empty(1, device=DEV)
    rc = lib.widek_batchnorm_train_fwd_noalloc(x.data_ptr(), x.data_ptr(), None, None, None, None, None, None,
                                               1, 1, 65537, 1, 0.1, 1e-5, N.F32,
                                               torch.cuda.current_stream().cuda_stream)
    assert rc == N.WIDEK_ERR_INVALID
    assert "fixed scratch" in N.last_error()
