"""wide_compiler (B200-native): fuse N identical models into one wide model
whose primitives run on hand-written sm_100a kernels (libwidek).

Drop-in for WideCompiler v0.6.0's public surface
(reference wide_compiler/__init__.py:1-234)::

    import wide_compiler
    wide = wide_compiler.compile(models, sample_input)      # TracedWideModel
    out = wide(wide_compiler.pack(inputs))                   # [B, N*C, ...]
    outs = wide_compiler.unpack(out, n=len(models))

The reference's benchmark subsystem is not shipped; as in the reference when
that subsystem is unavailable, the benchmark names are None.
"""
from .api import compile, WideBuilder, pack, unpack
from . import _torch_ops  # noqa: F401  (registers the torch.library operators widek::*)
from .core.config import WideConfig, get_default_config, set_default_config
from .core.registry import register, unregister, get_registry, list_registered
from .core.traced_wide import TracedWideModel, FunctionalOp, BinaryOp, print_trace
from .core.ensemble_util import pack_inputs, unpack_outputs
from .core.primitives import (WideLinear, WideConv1d, WideConv2d, WideConv3d, WideBatchNorm1d, WideBatchNorm2d,
                              WideLayerNorm, WideGroupNorm, WideInstanceNorm1d, WideInstanceNorm2d, WideEmbedding,
                              WideAttention, WideGRU, WideLSTM)

_HAS_BENCHMARK = False
benchmark_primitive = None
benchmark_multi = None
benchmark_all = None
benchmark_custom = None
list_benchmark_primitives = None
BenchmarkResult = None
SweepParams = None

__version__ = "0.6.0+b200"

__all__ = [
    'compile', 'WideBuilder', 'pack', 'unpack',
    'WideConfig', 'get_default_config', 'set_default_config',
    'register', 'unregister', 'get_registry', 'list_registered',
    'TracedWideModel', 'FunctionalOp', 'BinaryOp', 'print_trace', 'pack_inputs', 'unpack_outputs',
    'WideLinear', 'WideConv1d', 'WideConv2d', 'WideConv3d', 'WideBatchNorm1d', 'WideBatchNorm2d',
    'WideLayerNorm', 'WideGroupNorm', 'WideInstanceNorm1d', 'WideInstanceNorm2d', 'WideEmbedding',
    'WideAttention', 'WideGRU', 'WideLSTM',
    'benchmark_primitive', 'benchmark_multi', 'benchmark_all', 'benchmark_custom', 'list_benchmark_primitives',
    'BenchmarkResult', 'SweepParams',
]
