"""TracedWideModel: FX-trace one template model, build one wide stage per node.

Same construction and calling contract as the reference
(wide_compiler/core/traced_wide.py:270-534):

* ``from_models(models, sample_input)`` traces ``models[0]`` with
  ``torch.fx.symbolic_trace``; ``get_attr`` tensors of all N models are
  concatenated into ``_attr_*`` buffers; every ``call_module`` node whose type
  is in ``WIDE_BUILDERS`` becomes that Wide primitive (others run the
  template module unchanged on the N-first tensor); ``call_function`` /
  ``call_method`` nodes become ``BinaryOp`` / ``FunctionalOp`` stages.
* ``forward`` takes the channel-packed input [B, N*C, *S], runs the stages on
  the N-first layout [N, B, C, *S] and returns channel-packed [B, N*C, *S]
  (tuple outputs contribute their first element).

B200 path: the two layout changes at the boundary are single libwidek
transpose-copy kernels, and elementwise glue (ReLU/GELU/sigmoid/tanh/SiLU,
same-shape add/mul/sub/div) runs on libwidek kernels. Glue the kernels do not
cover (broadcasting against constants, arbitrary methods) executes the traced
torch call unchanged.
"""
from __future__ import annotations

import operator
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Tuple

import torch
import torch.fx as fx
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor

from .. import ops
from .ensemble_util import pack_inputs, unpack_outputs  # noqa: F401  (re-exported API)
from .primitives import (WideAttention, WideBatchNorm1d, WideBatchNorm2d, WideConv1d, WideConv2d, WideConv3d,
                         WideEmbedding, WideGroupNorm, WideGRU, WideInstanceNorm1d, WideInstanceNorm2d,
                         WideLayerNorm, WideLinear, WideLSTM)

WIDE_BUILDERS: Dict[str, Callable[[List[nn.Module]], nn.Module]] = {
    'Linear': WideLinear.from_modules,
    'Conv1d': WideConv1d.from_modules,
    'Conv2d': WideConv2d.from_modules,
    'Conv3d': WideConv3d.from_modules,
    'BatchNorm1d': WideBatchNorm1d.from_modules,
    'BatchNorm2d': WideBatchNorm2d.from_modules,
    'LayerNorm': WideLayerNorm.from_modules,
    'GroupNorm': WideGroupNorm.from_modules,
    'InstanceNorm1d': WideInstanceNorm1d.from_modules,
    'InstanceNorm2d': WideInstanceNorm2d.from_modules,
    'Embedding': WideEmbedding.from_modules,
    'MultiheadAttention': WideAttention.from_modules,
    'GRU': WideGRU.from_modules,
    'LSTM': WideLSTM.from_modules,
}


# ---------------------------------------------------------------------------
# Trace inspection helpers
# ---------------------------------------------------------------------------

@dataclass
class TraceNode:
    """One node of an FX graph, in execution order."""
    order: int
    op: str
    name: str
    target: Any
    args: Tuple
    kwargs: Dict


def analyze_trace(graph: fx.Graph) -> List[TraceNode]:
    return [TraceNode(i, n.op, n.name, n.target, n.args, dict(n.kwargs)) for i, n in enumerate(graph.nodes)]


def print_trace(traced: fx.GraphModule) -> str:
    lines = ["FX Trace:", "=" * 60]
    for n in traced.graph.nodes:
        if n.op == 'placeholder':
            lines.append(f"  [input] {n.name}")
        elif n.op == 'call_module':
            lines.append(f"  [module] {n.target}")
        elif n.op == 'call_function':
            lines.append(f"  [func] {getattr(n.target, '__name__', str(n.target))}")
        elif n.op == 'call_method':
            lines.append(f"  [method] .{n.target}()")
        elif n.op == 'get_attr':
            lines.append(f"  [attr] {n.target}")
        elif n.op == 'output':
            lines.append("  [output]")
    return "\n".join(lines)


# ---------------------------------------------------------------------------
# Glue stages
# ---------------------------------------------------------------------------

# Elementwise callables that map onto the libwidek unary kernel.
_UNARY_FUNCS = {
    F.relu: 'relu', torch.relu: 'relu',
    F.gelu: 'gelu',
    torch.sigmoid: 'sigmoid', F.sigmoid: 'sigmoid',
    torch.tanh: 'tanh', F.tanh: 'tanh',
    F.silu: 'silu',
}
_UNARY_MODULES = {nn.ReLU: 'relu', nn.GELU: 'gelu', nn.Sigmoid: 'sigmoid', nn.Tanh: 'tanh', nn.SiLU: 'silu'}


def _kernel_tensor(t: Any) -> bool:
    return isinstance(t, Tensor) and t.is_cuda and t.dtype in (torch.float32, torch.bfloat16, torch.float16)


class FunctionalOp(nn.Module):
    """Applies a traced function / method / passthrough module to N-first data.

    Known elementwise activations on CUDA tensors run on the libwidek unary
    kernel; anything else calls ``fn`` unchanged.
    """

    def __init__(self, fn: Callable, name: str = "", unary: Optional[str] = None):
        super().__init__()
        self.fn = fn
        self.name = name or getattr(fn, '__name__', 'func')
        self.unary = unary

    def forward(self, *args, **kwargs):
        if self.unary is not None and len(args) == 1 and _kernel_tensor(args[0]) and self._plain(kwargs):
            return ops.unary(args[0], self.unary)
        return self.fn(*args, **kwargs)

    def _plain(self, kwargs) -> bool:
        if not kwargs:
            return True
        # F.gelu(approximate='none') and inplace flags do not change the result.
        return all((k == 'approximate' and v == 'none') or (k == 'inplace') for k, v in kwargs.items())

    def __repr__(self):
        return f"FunctionalOp({self.name})"


_BINARY_TORCH = {
    'add': operator.add, 'mul': operator.mul, 'sub': operator.sub, 'div': operator.truediv,
    'matmul': operator.matmul,
}


class BinaryOp(nn.Module):
    """a op b for op in add / mul / sub / div / matmul (reference :189-211).

    Same-shape, same-dtype CUDA operands of add/mul/sub/div run on the libwidek
    binary kernel; other combinations (broadcasts, scalars, matmul) use the
    torch operator.
    """

    def __init__(self, op: str):
        super().__init__()
        if op not in _BINARY_TORCH:
            raise ValueError(f"Unknown op: {op}")
        self.op = op

    def forward(self, a, b):
        if (self.op != 'matmul' and _kernel_tensor(a) and _kernel_tensor(b) and a.shape == b.shape
                and a.dtype == b.dtype and a.device == b.device):
            return ops.binary(a, b, self.op)
        return _BINARY_TORCH[self.op](a, b)

    def __repr__(self):
        return f"BinaryOp({self.op})"


class GetAttrOp(nn.Module):
    """Placeholder stage for a ``get_attr`` node (the value is a buffer)."""

    def __init__(self, name: str):
        super().__init__()
        self.attr_name = name

    def forward(self, value: Tensor) -> Tensor:
        return value

    def __repr__(self):
        return f"GetAttrOp({self.attr_name})"


@dataclass
class WideStage:
    order: int
    name: str
    op_type: str
    target: str
    wide_op: nn.Module
    n: int
    num_inputs: int = 1


def _get_nested_attr(obj: Any, path: str) -> Any:
    for part in path.split('.'):
        obj = getattr(obj, part)
    return obj


def _function_stage(fn) -> nn.Module:
    if fn is operator.add or fn is torch.add:
        return BinaryOp('add')
    if fn is operator.mul or fn is torch.mul:
        return BinaryOp('mul')
    if fn is operator.sub:
        return BinaryOp('sub')
    if fn is operator.truediv:
        return BinaryOp('div')
    if fn is torch.matmul or fn is operator.matmul:
        return BinaryOp('matmul')
    return FunctionalOp(fn, getattr(fn, '__name__', str(fn)), unary=_UNARY_FUNCS.get(fn))


def _method_caller(method: str):
    def call(x, *args, **kwargs):
        return getattr(x, method)(*args, **kwargs)
    return call


_UNARY_METHODS = {'relu': 'relu', 'sigmoid': 'sigmoid', 'tanh': 'tanh'}


# ---------------------------------------------------------------------------
# TracedWideModel
# ---------------------------------------------------------------------------

class TracedWideModel(nn.Module):
    """N models fused into one stage graph built from an FX trace."""

    def __init__(self, n: int):
        super().__init__()
        self.n = n
        self.stages: nn.ModuleDict = nn.ModuleDict()
        self.stage_info: Dict[str, WideStage] = {}
        self._graph: Optional[fx.Graph] = None
        self._execution_order: List[str] = []
        self._node_args: Dict[str, Tuple] = {}
        self._node_kwargs: Dict[str, Dict] = {}
        self._input_name: str = 'x'
        self._output_name: str = ''
        self._attr_names: List[str] = []

    @classmethod
    def from_models(cls, models: List[nn.Module], sample_input: Tensor) -> 'TracedWideModel':
        n = len(models)
        wide = cls(n)
        template = models[0]
        try:
            traced = fx.symbolic_trace(template)
        except Exception as e:
            raise RuntimeError(f"FX tracing failed: {e}. Model may have dynamic control flow.")
        wide._graph = traced.graph

        # Pass 1: get_attr tensors of all N models -> concatenated buffers.
        for node in traced.graph.nodes:
            if node.op != 'get_attr':
                continue
            safe = f"_attr_{node.name.replace('.', '_')}"
            vals = []
            for m in models:
                try:
                    v = _get_nested_attr(m, node.target)
                except AttributeError:
                    vals = None
                    break
                if not isinstance(v, Tensor):
                    vals = None
                    break
                vals.append(v.data if isinstance(v, nn.Parameter) else v)
            if vals is not None and len(vals) == n:
                buf = torch.stack(vals) if vals[0].dim() == 0 else torch.cat(vals, dim=0)
                wide.register_buffer(safe, buf)
                wide._attr_names.append(node.name)
            else:
                try:
                    v = _get_nested_attr(template, node.target)
                except AttributeError:
                    continue
                if isinstance(v, Tensor):
                    wide.register_buffer(safe, v.clone())
                    wide._attr_names.append(node.name)

        # Pass 2: stages in execution order.
        for node in traced.graph.nodes:
            op = None
            if node.op == 'placeholder':
                wide._input_name = node.name
                continue
            if node.op == 'output':
                if node.args:
                    a = node.args[0]
                    wide._output_name = a.name if hasattr(a, 'name') else str(a)
                continue
            if node.op == 'get_attr':
                wide._execution_order.append(node.name)
                wide._node_args[node.name] = ()
                wide._node_kwargs[node.name] = {}
                continue
            if node.op == 'call_module':
                mods = [m.get_submodule(node.target) for m in models]
                tname = type(mods[0]).__name__
                if tname in WIDE_BUILDERS:
                    op = WIDE_BUILDERS[tname](mods)
                else:
                    unary = _UNARY_MODULES.get(type(mods[0]))
                    if isinstance(mods[0], nn.GELU) and getattr(mods[0], 'approximate', 'none') != 'none':
                        unary = None
                    op = FunctionalOp(lambda x, m=mods[0]: m(x), f"Passthrough({tname})", unary=unary)
            elif node.op == 'call_function':
                op = _function_stage(node.target)
            elif node.op == 'call_method':
                op = FunctionalOp(_method_caller(node.target), f".{node.target}()",
                                  unary=_UNARY_METHODS.get(node.target))
            if op is None:
                continue
            arg_names = [a.name if hasattr(a, 'name') else a for a in node.args]
            kw = {k: (v.name if hasattr(v, 'name') else v) for k, v in node.kwargs.items()}
            stage = WideStage(order=len(wide._execution_order), name=node.name, op_type=node.op,
                              target=str(node.target), wide_op=op, n=n, num_inputs=len(arg_names))
            wide.stages[node.name.replace('.', '_')] = op
            wide.stage_info[node.name] = stage
            wide._execution_order.append(node.name)
            wide._node_args[node.name] = tuple(arg_names)
            wide._node_kwargs[node.name] = kw
        return wide

    # -- execution ------------------------------------------------------------

    def _unpack(self, x: Tensor) -> Tensor:
        """[B, N*C, *S] -> [N, B, C, *S] (one transpose-copy kernel)."""
        b, nc = x.shape[0], x.shape[1]
        if nc % self.n != 0:
            raise ValueError(f"input dim 1 ({nc}) is not a multiple of N={self.n}")
        return ops.swap01(x.reshape(b, self.n, nc // self.n, *x.shape[2:]))

    def _pack(self, out: Tensor) -> Tensor:
        """[N, B, C, *S] -> [B, N*C, *S] (one transpose-copy kernel)."""
        n, b, c = out.shape[0], out.shape[1], out.shape[2]
        return ops.swap01(out).reshape(b, n * c, *out.shape[3:])

    def _run_stages(self, x: Tensor) -> Any:
        values: Dict[str, Any] = {self._input_name: x}
        for name in self._attr_names:
            buf = f"_attr_{name.replace('.', '_')}"
            if hasattr(self, buf):
                values[name] = getattr(self, buf)
        for name in self._execution_order:
            if name in self._attr_names or name not in self.stage_info:
                continue
            op = self.stages[name.replace('.', '_')]
            args = [values[a] if isinstance(a, str) and a in values else a for a in self._node_args[name]]
            kwargs = {k: (values[v] if isinstance(v, str) and v in values else v)
                      for k, v in self._node_kwargs.get(name, {}).items()}
            values[name] = op(*args, **kwargs)
        return values[self._output_name]

    def forward(self, x: Tensor) -> Tensor:
        out = self._run_stages(self._unpack(x))
        if isinstance(out, tuple):
            out = out[0]
        return self._pack(out)

    def summary(self) -> str:
        lines = [f"TracedWideModel: {self.n} models", "=" * 60, f"Stages: {len(self.stages)}",
                 f"Attrs: {len(self._attr_names)}", ""]
        total = 0
        for name in self._execution_order:
            if name in self._attr_names:
                buf = f"_attr_{name.replace('.', '_')}"
                if hasattr(self, buf):
                    lines.append(f"  [attr] {name}: {list(getattr(self, buf).shape)}")
                continue
            if name not in self.stage_info:
                continue
            op = self.stages[name.replace('.', '_')]
            p = sum(t.numel() for t in op.parameters())
            total += p
            args = ", ".join(str(a) for a in self._node_args[name])
            lines.append(f"  [{self.stage_info[name].order}] {name}({args}): {type(op).__name__} ({p:,} params)")
        lines += ["", f"Total: {total:,} params ({total // self.n:,} per model)"]
        return "\n".join(lines)


__all__ = ['TraceNode', 'analyze_trace', 'print_trace', 'FunctionalOp', 'BinaryOp', 'GetAttrOp', 'WideStage',
           'TracedWideModel', 'WIDE_BUILDERS']
