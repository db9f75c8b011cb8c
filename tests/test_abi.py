"""The C-ABI library: it loads without a GPU, exports exactly the entry
points include/widek.h declares, and rejects bad arguments with error codes
(argument checks run before any CUDA call, so no device is needed)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "widek.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"WIDEK_API\s+(?:int|int64_t|size_t|long long)\s+(widek_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "widek_linear_fwd" in syms and "widek_layernorm_fwd" in syms
    assert len(syms) >= 10


def test_library_exports_every_declared_symbol():
    from wide_compiler import _native
    lib = _native.load()
    for s in declared_symbols():
        assert hasattr(lib, s), f"libwidek.so does not export {s}"


def test_python_binding_covers_header():
    from wide_compiler import _native
    assert set(_native.SIGNATURES) == set(declared_symbols())


def test_version_and_error_reporting():
    from wide_compiler import _native as N
    lib = N.load()
    assert lib.widek_version() >= 100
    rc = lib.widek_linear_fwd(None, None, None, None, -1, 1, 1, 1, N.BF16, 0, None)
    assert rc == N.WIDEK_ERR_INVALID
    assert "negative" in N.last_error()
    rc = lib.widek_unary(None, None, 4, 99, N.F32, None)
    assert rc == N.WIDEK_ERR_INVALID
    rc = lib.widek_layernorm_fwd(None, None, None, None, 1, 1, 4, 1e-5, N.F32, None)
    assert rc == N.WIDEK_ERR_INVALID
    with pytest.raises(ValueError):
        N.check(rc, "layernorm")


def test_zero_sized_calls_are_noops():
    from wide_compiler import _native as N
    lib = N.load()
    assert lib.widek_linear_fwd(None, None, None, None, 0, 4, 4, 4, N.BF16, 0, None) == 0
    assert lib.widek_swap01(None, None, 0, 3, 16, None) == 0


def _header_param_counts():
    text = open(HEADER).read()
    out = {}
    for m in re.finditer(r"WIDEK_API\s+(?:int|int64_t|size_t|long long)\s+(widek_\w+)\s*\(([^)]*)\)", text, re.S):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else len(params.split(","))
    return out


def test_binding_argument_counts_match_header():
    from wide_compiler import _native
    counts = _header_param_counts()
    for name, argtypes in _native.SIGNATURES.items():
        assert len(argtypes) == counts[name], f"{name}: binding has {len(argtypes)} args, header {counts[name]}"


def test_mlp_chain_argument_checks():
    """widek_mlp_chain_fwd / _supported reject bad chains before any CUDA
    call; the size query answers on the host."""
    from wide_compiler import _native as N
    lib = N.load()
    I64, INT = ctypes.c_int64, ctypes.c_int
    dims = (I64 * 3)(64, 128, 64)
    acts = (INT * 2)(1, 0)
    assert lib.widek_mlp_chain_fwd(None, None, None, None, dims, acts, 0, 1, 1, 0, 0, N.F32, None) == N.WIDEK_ERR_INVALID
    assert lib.widek_mlp_chain_fwd(None, None, None, None, dims, acts, 2, 1, 1, 3, 0, N.F32, None) == N.WIDEK_ERR_INVALID
    bad = (INT * 2)(1, 7)
    assert lib.widek_mlp_chain_fwd(None, None, None, None, dims, bad, 2, 1, 1, 0, 0, N.F32, None) == N.WIDEK_ERR_INVALID
    assert lib.widek_mlp_chain_supported(dims, bad, 2, 1, 1, N.F32) == 0
    assert "activation" in N.last_error()
    assert lib.widek_mlp_chain_supported(dims, acts, 2, 100, 32, N.F32) == 1
    wide = (I64 * 2)(512, 512)          # 1 MB of fp32 weights: does not fit on chip
    assert lib.widek_mlp_chain_supported(wide, acts, 1, 1, 4, N.F32) == 0
    zero = (I64 * 2)(0, 8)
    assert lib.widek_mlp_chain_supported(zero, acts, 1, 1, 4, N.F32) == 0


def test_bounded_wait_probe_rejects_bad_limits():
    """Argument checks of the failure-path probe run on the host (nothing is
    launched), so they need no GPU."""
    from wide_compiler import _native as N
    lib = N.load()
    assert lib.widek_test_bounded_wait(0, None) == N.WIDEK_ERR_INVALID
    assert lib.widek_test_bounded_wait(2_000_000_000, None) == N.WIDEK_ERR_INVALID
    assert "limit" in N.last_error()


def test_backward_and_fused_entry_argument_checks():
    """The backward entries and the fused projection + LayerNorm reject bad
    arguments (and accept empty problems) before any CUDA call."""
    from wide_compiler import _native as N
    lib = N.load()
    P = 16                               # a stand-in pointer: never dereferenced on these paths
    assert lib.widek_linear_bwd_workspace(-1, 1, 1, 1, N.BF16) == -1
    ws = lib.widek_linear_bwd_workspace(2, 4, 8, 8, N.BF16)
    assert ws > 0
    assert lib.widek_linear_bwd(P, P, P, P, P, P, 2, 4, 8, 8, N.BF16, P, ws - 1, None) == N.WIDEK_ERR_INVALID
    assert "workspace" in N.last_error()
    assert lib.widek_linear_bwd(None, None, None, None, None, None, 0, 4, 8, 8, N.BF16, None, 0, None) == 0
    assert lib.widek_act_bwd(P, P, P, 4, 0, N.BF16, None) == N.WIDEK_ERR_INVALID
    assert lib.widek_transpose(P, P, 1, 2, 2, 9, None) == N.WIDEK_ERR_INVALID
    assert lib.widek_layernorm_bwd_workspace(-1, 1, 1) == -1
    assert lib.widek_layernorm_bwd(P, P, P, P, P, P, 1, 4, 2000, 1e-5, N.BF16, P, 1 << 20, None) == \
        N.WIDEK_ERR_UNSUPPORTED
    gws = lib.widek_groupnorm_bwd_workspace(2, 3, 8)
    assert gws > 0
    assert lib.widek_groupnorm_bwd(P, P, P, P, P, P, 2, 3, 5, 4, 2, 1e-5, N.BF16, P, gws, None) == \
        N.WIDEK_ERR_INVALID                                        # 5 channels in 2 groups
    assert lib.widek_groupnorm_bwd(P, P, P, P, P, P, 2, 3, 8, 4, 2, 1e-5, N.BF16, P, gws - 1, None) == \
        N.WIDEK_ERR_INVALID                                        # workspace too small
    assert lib.widek_batchnorm_bwd(P, P, P, None, None, P, P, P, 2, 3, 4, 5, 0, 1e-5, N.BF16, None) == \
        N.WIDEK_ERR_INVALID                                        # eval mode without running statistics
    assert lib.widek_batchnorm_bwd(None, None, None, None, None, None, None, None, 0, 3, 4, 5, 1, 1e-5, N.BF16,
                                   None) == 0
    assert lib.widek_linear_ln_fwd_ex(P, P, P, P, P, P, 2, 4, 8, 16, 4, 7, 0, 1e-5, N.BF16, None) == \
        N.WIDEK_ERR_INVALID                                        # unknown layout
    assert lib.widek_linear_ln_fwd_ex(P, P, P, P, P, P, 2, 4, 8, 16, 4, 0, 0, 1e-5, N.F32, None) == \
        N.WIDEK_ERR_UNSUPPORTED                                    # fp32: the caller runs the two ops
