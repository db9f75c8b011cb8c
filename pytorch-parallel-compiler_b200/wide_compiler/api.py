"""Public entry points: compile, WideBuilder, pack, unpack.

Same signatures, defaults, errors and debug output as the reference
(wide_compiler/api.py:36-325). The benchmark re-exports of the reference
(benchmark_primitive / benchmark_custom, api.py:332-404) belong to its
benchmark subsystem, which this package does not ship; they raise
NotImplementedError.
"""
from __future__ import annotations

import copy
import dataclasses
from typing import List, Optional, Union

import torch
import torch.nn as nn
from torch import Tensor

from .core.config import WideConfig, get_default_config
from .core.registry import get_registry


def compile(models: Union[nn.Module, List[nn.Module]], sample_input: Optional[Tensor] = None, *,
            n: Optional[int] = None, config: Optional[WideConfig] = None,
            compile_model: Optional[bool] = None, compile_mode: Optional[str] = None,
            validate: Optional[bool] = None, debug: Optional[bool] = None) -> nn.Module:
    """Fuses N models (or N fresh copies of one model) into a TracedWideModel.

    The returned model takes channel-packed input [B, N*C, ...] (see ``pack``)
    and runs every wide stage on the sm_100a kernels.
    """
    from .core.traced_wide import TracedWideModel

    cfg = config or get_default_config()
    for name, val in (('compile', compile_model), ('compile_mode', compile_mode), ('validate', validate),
                      ('debug', debug)):
        if val is not None:
            cfg = _with_override(cfg, name, val)

    if isinstance(models, nn.Module):
        if n is None:
            raise ValueError("n required when passing single model")
        template = models
        models = [_clone_model(template) for _ in range(n)]
    if not models:
        raise ValueError("models list is empty")

    if cfg.debug:
        print(f"[WideCompiler] Compiling {len(models)} models")
        print(f"[WideCompiler] Registry: {get_registry()}")
    if sample_input is None:
        raise ValueError("sample_input required for FX tracing. "
                         "Provide a sample input tensor with the expected shape.")

    wide_model = TracedWideModel.from_models(models, sample_input)
    if cfg.debug:
        print(f"[WideCompiler] Built model:\n{wide_model.summary()}")
    if cfg.validate:
        _validate_model(wide_model, models, sample_input, cfg)
    if cfg.compile:
        if cfg.debug:
            print(f"[WideCompiler] Compiling with mode={cfg.compile_mode}")
        wide_model = _graphed(wide_model)
    return wide_model


def _graphed(wide_model: nn.Module) -> nn.Module:
    """What ``compile=True`` maps to: the CUDA-graph executor. The stages
    already run as sm_100a kernels, so the remaining per-call cost is host
    dispatch and launches, which one graph replay removes; every
    compile_mode / compile_backend gets the same executor (the reference's
    torch.compile call, api.py:137-147, is not used)."""
    from .core.graphed import GraphedWideModel
    return GraphedWideModel(wide_model)


class WideBuilder:
    """Fluent builder: ``WideBuilder(models).with_sample(x).validate().build()``."""

    def __init__(self, models: Union[nn.Module, List[nn.Module]], n: Optional[int] = None):
        if isinstance(models, nn.Module):
            if n is None:
                raise ValueError("n required when passing single model")
            self._models = [_clone_model(models) for _ in range(n)]
        else:
            self._models = list(models)
        self._sample_input: Optional[Tensor] = None
        self._config = WideConfig.default()

    def with_sample(self, sample_input: Tensor) -> 'WideBuilder':
        self._sample_input = sample_input
        return self

    def with_config(self, config: WideConfig) -> 'WideBuilder':
        self._config = config
        return self

    def validate(self, enable: bool = True) -> 'WideBuilder':
        self._config = _with_override(self._config, 'validate', enable)
        return self

    def compile(self, mode: str = 'reduce-overhead') -> 'WideBuilder':
        self._config = _with_override(self._config, 'compile', True)
        self._config = _with_override(self._config, 'compile_mode', mode)
        return self

    def debug(self, enable: bool = True) -> 'WideBuilder':
        self._config = _with_override(self._config, 'debug', enable)
        return self

    def register(self, module_type: str, wide_class: type) -> 'WideBuilder':
        get_registry().register(module_type, wide_class)
        return self

    def build(self) -> nn.Module:
        from .core.traced_wide import TracedWideModel
        if self._sample_input is None:
            raise ValueError("sample_input required - call .with_sample()")
        if self._config.debug:
            print(f"[WideBuilder] Building from {len(self._models)} models")
        wide_model = TracedWideModel.from_models(self._models, self._sample_input)
        if self._config.validate:
            _validate_model(wide_model, self._models, self._sample_input, self._config)
        if self._config.compile:
            wide_model = _graphed(wide_model)
        return wide_model


def _clone_model(model: nn.Module) -> nn.Module:
    """Deep copy with freshly initialised parameters (reference api.py:244-252)."""
    cloned = copy.deepcopy(model)
    for m in cloned.modules():
        if hasattr(m, 'reset_parameters'):
            m.reset_parameters()
    return cloned


def _with_override(config: WideConfig, field: str, value) -> WideConfig:
    return dataclasses.replace(config, **{field: value})


def _validate_model(wide_model: nn.Module, models: List[nn.Module], sample_input: Tensor,
                    config: WideConfig) -> None:
    """Runs the wide model and the N models on the same sample; raises
    ValueError when max |diff| > validate_rtol (reference api.py:261-303)."""
    from .core.ensemble_util import pack_inputs, unpack_outputs
    n = len(models)
    inputs = [sample_input.clone() for _ in range(n)]
    packed = pack_inputs(inputs)
    wide_model.eval()
    for m in models:
        m.eval()
    with torch.no_grad():
        expected = [models[i](inputs[i]) for i in range(n)]
        actual = unpack_outputs(wide_model(packed), n)
    max_diff = max((expected[i] - actual[i]).abs().max().item() for i in range(n))
    if config.debug:
        print(f"[WideCompiler] Validation max_diff: {max_diff:.8f}")
    if max_diff > config.validate_rtol:
        raise ValueError(f"Validation failed: max_diff={max_diff:.8f} > rtol={config.validate_rtol}. "
                         "Wide model output differs from individual models.")


def pack(inputs: List[Tensor]) -> Tensor:
    """N inputs [B, F, ...] -> [B, N*F, ...]."""
    from .core.ensemble_util import pack_inputs
    return pack_inputs(inputs)


def unpack(output: Tensor, n: int) -> List[Tensor]:
    """[B, N*F, ...] -> N views [B, F, ...]."""
    from .core.ensemble_util import unpack_outputs
    return unpack_outputs(output, n)


def benchmark_primitive(name: str, preset: str = 'full', device: str = 'cuda', verbose: bool = True, **overrides):
    raise NotImplementedError("the reference's benchmark subsystem is not part of this package; "
                              "use bench.py at the repository root")


def benchmark_custom(model_class, input_shape, n_values, name: str = 'custom', device: str = 'cuda',
                     **model_kwargs):
    raise NotImplementedError("the reference's benchmark subsystem is not part of this package; "
                              "use bench.py at the repository root")


__all__ = ['compile', 'WideBuilder', 'pack', 'unpack', 'benchmark_primitive', 'benchmark_custom']
