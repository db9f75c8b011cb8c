"""wide_compiler.core: tracer, packing utilities, registry, config, primitives
(same exports as the reference's wide_compiler/core/__init__.py:1-85)."""
from .traced_wide import TracedWideModel, FunctionalOp, BinaryOp, print_trace
from .ensemble_util import pack_inputs, unpack_outputs
from .registry import (WideRegistry, get_registry, register, unregister, get_builder, build_wide,
                       list_registered)
from .config import WideConfig, get_default_config, set_default_config
from .primitives import (WideLinear, WideConv2d, WideConv1d, WideBatchNorm2d, WideBatchNorm1d, WideLayerNorm,
                         WideEmbedding)

__all__ = [
    'TracedWideModel', 'FunctionalOp', 'BinaryOp', 'print_trace',
    'pack_inputs', 'unpack_outputs',
    'WideRegistry', 'get_registry', 'register', 'unregister', 'get_builder', 'build_wide', 'list_registered',
    'WideConfig', 'get_default_config', 'set_default_config',
    'WideLinear', 'WideConv2d', 'WideConv1d', 'WideBatchNorm2d', 'WideBatchNorm1d', 'WideLayerNorm',
    'WideEmbedding',
]
