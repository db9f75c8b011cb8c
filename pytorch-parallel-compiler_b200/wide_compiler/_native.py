"""Loader for libwidek.so, the sm_100a kernels behind every wide primitive.

The library is a plain C-ABI shared object (``include/widek.h``); it is bound
with ctypes so that no torch C++ extension has to be compiled against a
particular torch build. Arguments are raw device pointers, sizes, dtype codes
and the current CUDA stream.

There is no fallback: if the library is missing or fails to load, every
primitive forward raises. Build it with
``python pytorch-parallel-compiler_b200/csrc/build.py`` (or
``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("WIDEK_LIB", os.path.join(_HERE, "_lib", "libwidek.so"))

WIDEK_OK = 0
WIDEK_ERR_INVALID = -1
WIDEK_ERR_UNSUPPORTED = -2
WIDEK_ERR_CUDA = -3
WIDEK_ERR_TIMEOUT = -4

# device error word codes (include/widek.h WIDEK_DEV_ERR_*)
DEV_ERR_GEMM_TIMEOUT, DEV_ERR_RNN_TIMEOUT, DEV_ERR_ATTN_TIMEOUT = 101, 102, 103
DEV_ERR_CONV_TIMEOUT, DEV_ERR_NORM_TIMEOUT, DEV_ERR_WAIT_PROBE, DEV_ERR_INDEX = 104, 105, 106, 110

F32, BF16, F16 = 0, 1, 2
ACT_NONE, ACT_RELU, ACT_GELU = 0, 1, 2

_DTYPE_CODES = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_dbl = ctypes.c_double

# name -> argtypes (restype is always c_int). Mirrors include/widek.h.
SIGNATURES = {
    "widek_version": [],
    "widek_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "widek_device_error": [ctypes.POINTER(ctypes.c_int)],
    "widek_test_bounded_wait": [ctypes.c_uint64, _c_void_p],
    "widek_linear_fwd": [_c_void_p] * 4 + [_i64] * 4 + [_int, _int, _c_void_p],
    "widek_linear_fwd_ex": [_c_void_p] * 4 + [_i64] * 5 + [_int] * 4 + [_c_void_p],
    "widek_linear_fwd_simt": [_c_void_p] * 4 + [_i64] * 4 + [_int, _int, _c_void_p],
    "widek_linear_set_variant": [_int],
    "widek_attention_set_variant": [_int],
    "widek_conv_set_variant": [_int],
    "widek_rnn_set_variant": [_int],
    "widek_launch_count": [],
    "widek_layernorm_fwd": [_c_void_p] * 4 + [_i64] * 3 + [_dbl, _int, _c_void_p],
    "widek_layernorm_fwd_ex": [_c_void_p] * 4 + [_i64] * 4 + [_dbl, _int, _c_void_p],
    "widek_swap01": [_c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p],
    "widek_pack": [ctypes.POINTER(_c_void_p), _i64, _c_void_p, _i64, _i64, _c_void_p],
    "widek_copy2d": [_c_void_p, _i64, _c_void_p, _i64, _i64, _i64, _c_void_p],
    "widek_unary": [_c_void_p, _c_void_p, _i64, _int, _int, _c_void_p],
    "widek_binary": [_c_void_p, _c_void_p, _c_void_p, _i64, _int, _int, _c_void_p],
    "widek_batchnorm_fwd": [_c_void_p] * 6 + [_i64] * 4 + [_dbl, _int, _c_void_p],
    "widek_batchnorm_train_workspace": [_i64] * 4,
    "widek_batchnorm_train_fwd": [_c_void_p] * 9 + [ctypes.c_size_t] + [_i64] * 4 + [_dbl, _dbl, _int, _c_void_p],
    "widek_batchnorm_train_fwd_noalloc": [_c_void_p] * 8 + [_i64] * 4 + [_dbl, _dbl, _int, _c_void_p],
    "widek_groupnorm_fwd": [_c_void_p] * 6 + [_i64] * 5 + [_dbl, _int, _c_void_p],
    "widek_embedding_fwd": [_c_void_p] * 3 + [_i64] * 4 + [_int, _c_void_p],
    "widek_gru_recurrence": [_c_void_p] * 6 + [_i64] * 4 + [_int, _c_void_p],
    "widek_lstm_recurrence": [_c_void_p] * 8 + [_i64] * 4 + [_int, _c_void_p],
    "widek_gru_fwd": [_c_void_p] * 8 + [ctypes.POINTER(_i64), _c_void_p, ctypes.c_size_t] + [_i64] * 5
                     + [_int, _c_void_p],
    "widek_lstm_fwd": [_c_void_p] * 10 + [ctypes.POINTER(_i64), _c_void_p, ctypes.c_size_t] + [_i64] * 5
                      + [_int, _c_void_p],
    "widek_gru_fwd_ex": [_c_void_p] * 8 + [ctypes.POINTER(_i64), _c_void_p, ctypes.c_size_t] + [_i64] * 5
                        + [_int] * 3 + [_c_void_p],
    "widek_lstm_fwd_ex": [_c_void_p] * 10 + [ctypes.POINTER(_i64), _c_void_p, ctypes.c_size_t] + [_i64] * 5
                         + [_int] * 3 + [_c_void_p],
    "widek_rnn_workspace": [_int] + [_i64] * 4 + [_int],
    "widek_conv_pack_weight": [_c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _c_void_p],
    "widek_conv_workspace": [_i64] * 6 + [_int],
    "widek_conv_packed_weight_elems": [_i64] * 3,
    "widek_conv_fwd": [_c_void_p] * 9 + [ctypes.c_size_t, ctypes.POINTER(_i64), _int, _int, _int, _c_void_p],
    "widek_conv_fwd_ex": [_c_void_p] * 9 + [ctypes.c_size_t, ctypes.POINTER(_i64)] + [_int] * 6 + [_c_void_p],
    "widek_conv_layouts_supported": [ctypes.POINTER(_i64)] + [_int] * 5,
    "widek_conv_path": [ctypes.POINTER(_i64)] + [_int] * 5,
    "widek_mlp_chain_fwd": [_c_void_p, _c_void_p, ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p),
                            ctypes.POINTER(_i64), ctypes.POINTER(_int), _int, _i64, _i64, _int, _int, _int,
                            _c_void_p],
    "widek_mlp_chain_supported": [ctypes.POINTER(_i64), ctypes.POINTER(_int), _int, _i64, _i64, _int],
    "widek_mlp_chain_set_variant": [_int],
    "widek_attention_fwd": [_c_void_p] * 4 + [_i64] * 9 + [_int, _c_void_p, _int, ctypes.POINTER(_i64), _dbl,
                                                          _int, _c_void_p],
    "widek_transpose": [_c_void_p, _c_void_p, _i64, _i64, _i64, _int, _c_void_p],
    "widek_linear_ln_fwd_ex": [_c_void_p] * 6 + [_i64] * 5 + [_int, _int, _dbl, _int, _c_void_p],
    "widek_batchnorm_bwd": [_c_void_p] * 8 + [_i64] * 4 + [_int, _dbl, _int, _c_void_p],
    "widek_groupnorm_bwd_workspace": [_i64] * 3,
    "widek_groupnorm_bwd": [_c_void_p] * 6 + [_i64] * 5 + [_dbl, _int, _c_void_p, _i64, _c_void_p],
    "widek_linear_bwd_workspace": [_i64] * 4 + [_int],
    "widek_linear_bwd": [_c_void_p] * 6 + [_i64] * 4 + [_int, _c_void_p, _i64, _c_void_p],
    "widek_act_bwd": [_c_void_p] * 3 + [_i64, _int, _int, _c_void_p],
    "widek_layernorm_bwd_workspace": [_i64] * 3,
    "widek_layernorm_bwd": [_c_void_p] * 6 + [_i64] * 3 + [_dbl, _int, _c_void_p, _i64, _c_void_p],
}
RESTYPES = {"widek_batchnorm_train_workspace": ctypes.c_size_t, "widek_conv_workspace": ctypes.c_size_t,
            "widek_rnn_workspace": ctypes.c_size_t, "widek_conv_packed_weight_elems": _i64,
            "widek_launch_count": ctypes.c_longlong, "widek_linear_bwd_workspace": _i64,
            "widek_layernorm_bwd_workspace": _i64, "widek_groupnorm_bwd_workspace": _i64}


class WideKernelError(RuntimeError):
    """A libwidek entry point reported a failure."""


_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Loads libwidek.so once and binds every declared entry point."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"wide_compiler: native kernel library not found at {LIB_PATH}. "
                "Build it with `python pytorch-parallel-compiler_b200/csrc/build.py`; "
                "there is no non-CUDA implementation of the wide primitives.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = RESTYPES.get(name, ctypes.c_int)
        _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    """The loaded library (or, while a :class:`LaunchTimer` is active, a view
    of it that brackets every compute entry point with CUDA events)."""
    base = _lib if _lib is not None else load()
    return base if _timer is None else _timer.view(base)


# Entry points that launch work (everything else is a query or a setter).
_LAUNCHING = frozenset(n for n in SIGNATURES if n.endswith(("_fwd", "_fwd_ex", "_fwd_simt", "_recurrence", "_bwd"))
                       or n in ("widek_swap01", "widek_pack", "widek_copy2d", "widek_unary", "widek_binary",
                                "widek_conv_pack_weight", "widek_batchnorm_train_fwd_noalloc", "widek_transpose"))

_timer: Optional["LaunchTimer"] = None


class LaunchTimer:
    """Times every launching entry point called while it is active, with a
    pair of CUDA events on torch's current stream (the stream the library
    launches on) around the call. ``summary()`` gives, per entry point, the
    number of calls and their mean and total device time in milliseconds.
    Used by bench.py to measure the dominant kernel inside its timed region;
    a CUDA-graph replay launches nothing through the library and is not
    seen."""

    def __init__(self):
        self.events = {}
        self._wrapped = {}
        self._base = None

    def __enter__(self):
        global _timer
        if _timer is not None:
            raise RuntimeError("LaunchTimer: another timer is active")
        _timer = self
        return self

    def __exit__(self, *exc):
        global _timer
        _timer = None
        return False

    def view(self, base):
        self._base = base
        return self

    def __getattr__(self, name):
        fn = getattr(self._base, name)
        if name not in _LAUNCHING:
            return fn
        w = self._wrapped.get(name)
        if w is None:
            def w(*args, _fn=fn, _name=name):
                s = torch.cuda.current_stream()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                rc = _fn(*args)
                e1.record(s)
                self.events.setdefault(_name, []).append((e0, e1))
                return rc
            self._wrapped[name] = w
        return w

    def summary(self) -> dict:
        """{entry point: {"calls", "mean_ms", "total_ms"}} (synchronizes)."""
        torch.cuda.synchronize()
        out = {}
        for name, evs in self.events.items():
            ts = [a.elapsed_time(b) for a, b in evs]
            out[name] = {"calls": len(ts), "mean_ms": sum(ts) / len(ts), "total_ms": sum(ts)}
        return out


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().widek_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc == WIDEK_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (WIDEK_ERR_INVALID, WIDEK_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise WideKernelError(msg)


_replayed_launches = 0


def note_replayed_launches(n: int) -> None:
    """Counts n library kernels launched by replaying a recorded CUDA graph
    (the launches were counted once when the graph was recorded)."""
    global _replayed_launches
    _replayed_launches += n


def launch_count() -> int:
    """Kernel launches the library has issued in this process, including
    those run by replays of the CUDA-graph executor's recorded graphs."""
    return int(lib().widek_launch_count()) + _replayed_launches


def device_error() -> int:
    """Synchronizes, returns and clears the device-side error word."""
    code = ctypes.c_int(0)
    check(lib().widek_device_error(ctypes.byref(code)), "widek_device_error")
    return code.value


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"wide_compiler kernels support float32/bfloat16/float16, got {t.dtype}") from None


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> int:
    """Handle of torch's current stream on `device` (the raw query when torch
    has it: no Stream object is built per launch)."""
    if _raw_stream is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def require_cuda(*tensors: Optional[torch.Tensor], what: str) -> torch.device:
    """Every tensor must be a CUDA tensor on one device; returns that device."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                f"{what}: wide_compiler runs the wide primitives only on CUDA (sm_100a) tensors; "
                f"got a tensor on {t.device}. Move the module and its inputs to a B200 GPU.")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{what}: tensors on different devices ({dev} and {t.device})")
    if dev is None:
        raise RuntimeError(f"{what}: no tensor arguments")
    return dev
