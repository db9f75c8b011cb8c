"""Helpers shared by the GPU parity tests."""
import torch

# fp32 contract (TF32 off): rtol 1e-3 / atol 1e-4 against the fp32 reference.
FP32_TOL = dict(rtol=1e-3, atol=1e-4)
# bf16/f16 contract: rtol 2e-2 against an fp32 (here fp64) reference computed
# from the same (rounded) inputs; atol scaled to the output's magnitude so that
# outputs near zero are judged by the storage precision.
LOWP_RTOL = 2e-2


def assert_lowp_close(actual: torch.Tensor, expected: torch.Tensor, rtol: float = LOWP_RTOL, atol_frac: float = 1e-2):
    e = expected.double().cpu()
    a = actual.double().cpu()
    scale = float(e.abs().max()) if e.numel() else 1.0
    torch.testing.assert_close(a, e, rtol=rtol, atol=atol_frac * max(scale, 1e-6))


def assert_fp32_close(actual: torch.Tensor, expected: torch.Tensor):
    torch.testing.assert_close(actual.double().cpu(), expected.double().cpu(), **FP32_TOL)


def no_device_error():
    from wide_compiler import _native
    assert _native.device_error() == 0


def kernels_run(fn):
    """Names of the CUDA kernels ``fn`` launches (torch profiler)."""
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}
