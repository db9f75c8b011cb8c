"""WideConfig: options of wide_compiler.compile / WideBuilder.

Same fields, defaults and presets as the reference's configuration
(wide_compiler/core/config.py:17-109). One deliberate difference: in the
reference the ``debug`` preset classmethod (config.py:94) shadows the
``debug`` dataclass field, so ``WideConfig().debug`` is a bound method (always
truthy) and ``compile`` always prints its debug lines. Here ``WideConfig.debug``
still works as the preset constructor when read on the class, while instances
carry a real boolean field.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, Literal, Optional

_COMPILE_MODES = ('default', 'reduce-overhead', 'max-autotune')
_PRECISIONS = ('fp32', 'fp16', 'bf16')


@dataclass
class WideConfig:
    """Configuration for building a wide model.

    n: number of fused models (None: taken from the model list).
    compile: wrap the result in the CUDA-graph executor
        (``core.graphed.GraphedWideModel``); compile_mode / compile_backend /
        compile_options are validated and recorded (every mode gets the
        same executor; no torch.compile).
    precision, allow_tf32: recorded for compatibility (the kernels compute in
        fp32 whatever the storage dtype).
    validate / validate_rtol / validate_atol: compare the wide model against
        the N source models after building (max |diff| <= validate_rtol).
    fallback_passthrough, strict_architecture, profile: recorded for
        compatibility.
    debug: print build information.
    """

    n: Optional[int] = None
    compile: bool = False
    compile_mode: Literal['default', 'reduce-overhead', 'max-autotune'] = 'reduce-overhead'
    compile_backend: str = 'inductor'
    compile_options: Dict[str, Any] = field(default_factory=dict)
    precision: Literal['fp32', 'fp16', 'bf16'] = 'fp32'
    allow_tf32: bool = True
    validate: bool = False
    validate_rtol: float = 1e-3
    validate_atol: float = 1e-5
    fallback_passthrough: bool = True
    strict_architecture: bool = True
    debug: bool = False
    profile: bool = False

    def __post_init__(self):
        if self.compile_mode not in _COMPILE_MODES:
            raise ValueError(f"compile_mode must be one of {_COMPILE_MODES}")
        if self.precision not in _PRECISIONS:
            raise ValueError(f"precision must be one of {_PRECISIONS}")

    @classmethod
    def default(cls) -> 'WideConfig':
        return cls()

    @classmethod
    def fast(cls) -> 'WideConfig':
        return cls(compile=True, compile_mode='reduce-overhead', allow_tf32=True, validate=False)

    @classmethod
    def safe(cls) -> 'WideConfig':
        return cls(compile=False, validate=True, strict_architecture=True)


def _debug_preset(cls) -> WideConfig:
    return cls(compile=False, validate=True, debug=True, fallback_passthrough=False)


class _DebugAttr:
    """``WideConfig.debug()`` builds the debug preset; ``cfg.debug`` is a bool."""

    def __get__(self, obj, objtype=None):
        if obj is None:
            return lambda: _debug_preset(objtype)
        return obj.__dict__.get('debug', False)

    def __set__(self, obj, value):
        obj.__dict__['debug'] = value


WideConfig.debug = _DebugAttr()

_default_config: Optional[WideConfig] = None


def get_default_config() -> WideConfig:
    global _default_config
    if _default_config is None:
        _default_config = WideConfig.default()
    return _default_config


def set_default_config(config: WideConfig) -> None:
    global _default_config
    _default_config = config


__all__ = ['WideConfig', 'get_default_config', 'set_default_config']
