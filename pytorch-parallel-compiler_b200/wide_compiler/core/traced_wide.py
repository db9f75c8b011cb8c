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

from .. import _derived, ops
from .ensemble_util import pack_inputs, unpack_outputs  # noqa: F401  (re-exported API)
from .primitives import (WideAttention, WideBatchNorm1d, WideBatchNorm2d, WideConv1d, WideConv2d, WideConv3d,
                         WideEmbedding, WideGroupNorm, WideGRU, WideInstanceNorm1d, WideInstanceNorm2d,
                         WideLayerNorm, WideLinear, WideLSTM)

# A chain of small Linears runs as one launch (one CTA per model, CUDA-core
# FMAs) up to this many multiply-adds for bf16/f16 (4x for fp32, whose
# per-layer path is CUDA-core too); above it the per-layer tcgen05 GEMMs win.
CHAIN_MAX_MACS = 1 << 25

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

    def forward_packed(self, *args, **kwargs):
        """Elementwise activations give the same values in any layout, so they
        run on the packed boundary layout as is; other functions decline."""
        if self.unary is not None and len(args) == 1 and _kernel_tensor(args[0]) and self._plain(kwargs):
            return ops.unary(args[0], self.unary)
        return None

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

    def forward_packed(self, a, b):
        """On the packed boundary layout: two packed operands of one shape
        (elementwise, so layout-independent), or a packed operand and a Python
        number; anything that broadcasts declines."""
        if self.op == 'matmul':
            return None
        if isinstance(a, Tensor) and isinstance(b, Tensor):
            return self.forward(a, b) if a.shape == b.shape else None
        if isinstance(a, (int, float)) or isinstance(b, (int, float)):
            return _BINARY_TORCH[self.op](a, b)
        return None

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


def _bn_fold(bn: nn.Module):
    """Eval-mode BatchNorm as a per-channel scale/shift (fp32):
    scale = w / sqrt(running_var + eps), shift = b - running_mean * scale."""
    rv = bn.running_var.float()
    scale = torch.rsqrt(rv + bn.eps)
    if bn.weight is not None:
        scale = scale * bn.weight.float()
    shift = -bn.running_mean.float() * scale
    if bn.bias is not None:
        shift = shift + bn.bias.float()
    return scale, shift


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

class _Laid:
    """A value kept in a layout other than N-first until a consumer needs the
    N-first tensor: the packed model input [B, N*C, *S] (fused conv groups
    read it directly), the packed model output written by the last fused
    conv, or a channels-last conv output consumed only by the next fused
    conv. `std` caches the N-first tensor once it has been made."""
    __slots__ = ('t', 'layout', 'std')

    def __init__(self, t: Tensor, layout: int):
        self.t, self.layout, self.std = t, layout, None


class _Decline:
    """Marker: an argument that rules out the packed-layout call."""


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
        # Cross-stage fusion (Linear+act, Conv+BN[+act|+residual[+act]]);
        # the plan is built on the first forward.
        self.fuse: bool = True
        self._fusion: Optional[Dict[str, Any]] = None

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

    # -- cross-stage fusion ----------------------------------------------------

    def _consumers(self) -> Dict[str, List[str]]:
        cons: Dict[str, List[str]] = {}
        for name in self._execution_order:
            refs = list(self._node_args.get(name, ())) + list(self._node_kwargs.get(name, {}).values())
            for a in refs:
                if isinstance(a, str):
                    cons.setdefault(a, []).append(name)
        cons.setdefault(self._output_name, []).append('<output>')
        return cons

    def _build_fusion_plan(self) -> Dict[str, Any]:
        """Groups of single-consumer chains executed as one kernel:
        Linear -> act; Conv -> BatchNorm(eval) [-> act | -> add(residual) [-> act]].
        Returns {last_node: group} and the set of nodes folded into groups."""
        from ..ops import ACT_GELU, ACT_RELU
        cons = self._consumers()
        acts = {'relu': ACT_RELU, 'gelu': ACT_GELU}
        groups: Dict[str, Dict[str, Any]] = {}
        folded = set()

        def only_consumer(name):
            c = cons.get(name, [])
            return c[0] if len(c) == 1 and c[0] in self.stage_info and c[0] not in folded else None

        def op_of(name):
            return self.stages[name.replace('.', '_')]

        def unary_act(name):
            o = op_of(name)
            if isinstance(o, FunctionalOp) and o.unary in acts and len(self._node_args[name]) == 1 \
                    and o._plain(self._node_kwargs.get(name, {})):
                return acts[o.unary]
            return None

        for name in self._execution_order:
            if name not in self.stage_info or name in folded:
                continue
            op = op_of(name)
            if isinstance(op, WideLinear) and len(self._node_args[name]) == 1:
                nxt = only_consumer(name)
                if nxt is not None and unary_act(nxt) is not None:
                    groups[nxt] = {'kind': 'linear', 'nodes': [name, nxt], 'head': name, 'act': unary_act(nxt)}
                    folded.update([name])
                continue
            if isinstance(op, (WideConv1d, WideConv2d)) and len(self._node_args[name]) == 1:
                bn = only_consumer(name)
                if bn is None or not isinstance(op_of(bn), (WideBatchNorm1d, WideBatchNorm2d)):
                    continue
                g = {'kind': 'conv', 'nodes': [name, bn], 'head': name, 'bn': bn, 'act': 0,
                     'residual': None, 'residual_first': False}
                tail = bn
                nxt = only_consumer(bn)
                if nxt is not None and unary_act(nxt) is not None:
                    g['act'] = unary_act(nxt)
                    g['nodes'].append(nxt)
                    tail = nxt
                elif nxt is not None and isinstance(op_of(nxt), BinaryOp) and op_of(nxt).op == 'add' \
                        and not self._node_kwargs.get(nxt):
                    a0, a1 = self._node_args[nxt]
                    other = a1 if a0 == bn else a0
                    if isinstance(other, str) and other != bn:
                        g['residual'] = other
                        g['nodes'].append(nxt)
                        tail = nxt
                        after = only_consumer(nxt)
                        if after is not None and unary_act(after) is not None:
                            g['act'] = unary_act(after)
                            g['residual_first'] = True
                            g['nodes'].append(after)
                            tail = after
                groups[tail] = g
                folded.update(g['nodes'][:-1])
        self._plan_linear_chains(groups, folded, cons, op_of)
        self._plan_attn_ln(groups, folded, cons, op_of)
        by_head = {g['head']: g for g in groups.values()}
        return {'groups': groups, 'folded': folded, 'consumers': cons, 'by_head': by_head}

    def _plan_attn_ln(self, groups, folded, cons, op_of) -> None:
        """Self-attention (one input, no mask) whose output is read only by a
        WideLayerNorm of the same width: the LayerNorm runs in the output
        projection's epilogue (attention out-projection + LN; reference
        wide_attention.py:233-236 then wide_layernorm.py:62-65). A traced
        nn.MultiheadAttention returns (output, weights): the output reaches
        the LayerNorm through getitem 0, and getitems of the weights that
        nothing reads fold into the group."""
        order = {nm: i for i, nm in enumerate(self._execution_order)}
        for name in self._execution_order:
            if name not in self.stage_info or name in folded or name in groups:
                continue
            op = op_of(name)
            if not isinstance(op, WideAttention):
                continue
            args = self._node_args[name]
            kw = self._node_kwargs.get(name, {})
            if not args or not isinstance(args[0], str) or any(a != args[0] for a in args):
                continue
            if any(k not in ('is_causal', 'need_weights') for k in kw) or \
                    not isinstance(kw.get('is_causal', False), bool):
                continue
            users = cons.get(name, [])
            path = [name]
            if len(users) == 1 and users[0] in self.stage_info and isinstance(op_of(users[0]), WideLayerNorm):
                ln = users[0]
            else:
                items: Dict[Any, List[str]] = {}
                ok = bool(users)
                for u in users:
                    uo = op_of(u) if u in self.stage_info else None
                    ua = self._node_args.get(u, ())
                    if not (isinstance(uo, FunctionalOp) and uo.fn is operator.getitem and len(ua) == 2
                            and ua[0] == name and not isinstance(ua[1], str) and u not in folded
                            and not self._node_kwargs.get(u)):
                        ok = False
                        break
                    items.setdefault(ua[1], []).append(u)
                if not ok or len(items.get(0, [])) != 1:
                    continue
                dead = [u for key, us in items.items() if key != 0 for u in us]
                if any(cons.get(u) for u in dead):
                    continue
                g0 = items[0][0]
                nxt = cons.get(g0, [])
                if len(nxt) != 1 or nxt[0] not in self.stage_info:
                    continue
                ln = nxt[0]
                path += [g0] + dead
            lop = op_of(ln)
            if ln in folded or not isinstance(lop, WideLayerNorm) or len(self._node_args[ln]) != 1 \
                    or self._node_kwargs.get(ln) or lop.n != op.n or lop.normalized_shape != op.d_model:
                continue
            if self._node_args[ln][0] != path[-1 if len(path) == 1 else 1]:
                continue
            nodes = sorted(path, key=order.get) + [ln]
            groups[ln] = {'kind': 'attn_ln', 'nodes': nodes, 'head': name, 'ln': ln,
                          'is_causal': bool(kw.get('is_causal', False))}
            folded.update(nodes[:-1])

    def _plan_linear_chains(self, groups, folded, cons, op_of) -> None:
        """Merges runs of WideLinear[+act] segments, each the only consumer
        of the previous one's output, into 'chain' groups (one libwidek
        launch for the whole run, boundary pack/unpack fused when the run
        starts at the model input or ends at the model output). A chain has
        two or more layers, or one layer that touches the model boundary."""
        lin_groups = {g['head']: (list(g['nodes']), tail, g['act'])
                      for tail, g in groups.items() if g['kind'] == 'linear'}
        segs = {}          # head -> (nodes, tail, act)
        for name in self._execution_order:
            if name not in self.stage_info or not isinstance(op_of(name), WideLinear) \
                    or len(self._node_args[name]) != 1 or self._node_kwargs.get(name):
                continue
            if name in lin_groups:
                segs[name] = lin_groups[name]
            elif name not in folded:
                segs[name] = ([name], name, 0)
        seg_by_tail = {s[1]: h for h, s in segs.items()}

        def next_seg(tail):
            c = cons.get(tail, [])
            if len(c) == 1 and c[0] in segs and self._node_args[c[0]][0] == tail:
                return c[0]
            return None

        for head in [h for h in self._execution_order if h in segs]:
            src = self._node_args[head][0]
            if src in seg_by_tail and next_seg(src) == head:
                continue           # inside the chain that starts further up
            layers, acts, nodes = [], [], []
            cur = head
            while cur is not None:
                seg_nodes, tail, act = segs[cur]
                layers.append(cur)
                acts.append(act)
                nodes.extend(seg_nodes)
                cur = next_seg(tail)
            tail = nodes[-1]
            boundary = self._node_args[head][0] == self._input_name or \
                (tail == self._output_name and cons.get(tail) == ['<output>'])
            if len(layers) < 2 and not boundary:
                continue
            for t in [t for t, g in groups.items() if g['kind'] == 'linear' and g['head'] in layers]:
                del groups[t]
            groups[tail] = {'kind': 'chain', 'nodes': nodes, 'head': head, 'layers': layers, 'acts': acts}
            folded.update(nodes[:-1])

    def _run_chain(self, g: Dict[str, Any], xv: Any):
        """A 'chain' group: one widek_mlp_chain_fwd launch when the chain fits
        the kernel (and is small enough that one CTA per model beats the
        per-layer tensor-core GEMMs), else one fused Linear+act per layer."""
        from .. import ops
        mods = g.get('mods')
        if mods is None:
            mods = g['mods'] = [self.stages[name.replace('.', '_')] for name in g['layers']]
        ws = [m.weight for m in mods]
        bs = [m.bias for m in mods]
        n = mods[0].n
        t = xv.t if isinstance(xv, _Laid) else xv
        packed_in = isinstance(xv, _Laid) and xv.layout == ops.LAYOUT_PACKED
        tail = g['nodes'][-1]
        at_output = tail == self._output_name and self._fusion['consumers'].get(tail) == ['<output>']
        if packed_in and t.dim() == 3 and t.shape[1] % n == 0:
            # packed [B, N*T, K] rows: the per-layer GEMMs read the packed
            # input and write the packed output in place (no unpack / pack)
            h, in_p = t, True
            for i, (w, b, act) in enumerate(zip(ws, bs, g['acts'])):
                out_p = at_output and i == len(ws) - 1
                h = ops.linear_layout(h, w, b, act, in_p, out_p) if (in_p or out_p) else ops.linear(h, w, b, act=act)
                in_p = False
            return _Laid(h, ops.LAYOUT_PACKED) if at_output else h
        if packed_in and t.dim() == 2:
            x_in, in_l, batch_shape = t, ops.LAYOUT_PACKED, (t.shape[0],)
        else:
            x_in = self._std(xv)
            batch_shape = tuple(x_in.shape[1:-1])
            x_in, in_l = x_in.reshape(n, -1, x_in.shape[-1]), ops.LAYOUT_NFIRST
        rows = 1
        for s in batch_shape:
            rows *= s
        macs = n * rows * sum(w.shape[1] * w.shape[2] for w in ws)
        limit = CHAIN_MAX_MACS * (4 if t.dtype == torch.float32 else 1)
        if x_in.dtype == ws[0].dtype and macs <= limit:
            out_l = ops.LAYOUT_PACKED if at_output and len(batch_shape) == 1 else ops.LAYOUT_NFIRST
            y = ops.mlp_chain(x_in, ws, bs, g['acts'], n, in_layout=in_l, out_layout=out_l)
            if y is not None:
                if out_l == ops.LAYOUT_PACKED:
                    return _Laid(y, out_l)
                return y.reshape(n, *batch_shape, y.shape[-1])
        h = self._std(xv)
        for w, b, act in zip(ws, bs, g['acts']):
            h = ops.linear(h, w, b, act=act)
        return h

    def _group_ready(self, g: Dict[str, Any], values: Dict[str, Any]) -> bool:
        """Whether a fused group can run now (eval-mode BatchNorm with
        running statistics, CUDA input, residual available)."""
        x = values.get(self._node_args[g['head']][0])
        t = x.t if isinstance(x, _Laid) else x
        if not isinstance(t, Tensor) or not t.is_cuda:
            return False
        if g['kind'] in ('linear', 'chain'):
            return True
        if g['kind'] == 'attn_ln':
            op = self.stages[g['head'].replace('.', '_')]
            return not (op.training and op.dropout > 0.0)
        bn_mod = self.stages[g['bn'].replace('.', '_')].op
        if bn_mod.training or bn_mod.running_mean is None or bn_mod.running_var is None:
            return False
        if g['residual'] is not None:
            r = values.get(g['residual'])
            r = r.t if isinstance(r, _Laid) else r
            if not isinstance(r, Tensor) or r.dtype != t.dtype or r.device != t.device:
                return False
        return True

    def _conv_params(self, op):
        if isinstance(op, WideConv2d):
            return op.grouped_conv.weight, op.grouped_conv.bias, op.stride, op.padding, op.dilation
        w, b = op._params()
        return w, b, (op.stride,), (op.padding,), (op.dilation,)

    def _next_conv_group(self, g: Dict[str, Any]) -> Optional[Dict[str, Any]]:
        """The fused conv group whose input is g's output, when that group
        is the output's only consumer."""
        tail = g['nodes'][-1]
        cons = self._fusion.get('consumers', {}).get(tail, [])
        if len(cons) != 1:
            return None
        head_group = self._fusion.get('by_head', {}).get(cons[0])
        if head_group is None or head_group['kind'] != 'conv':
            return None
        if self._node_args[head_group['head']][0] != tail or head_group['residual'] == tail:
            return None
        return head_group

    def _run_group(self, g: Dict[str, Any], values: Dict[str, Any]):
        """Executes a fused group; returns None when it cannot run fused
        (e.g. BatchNorm in training mode), in which case the nodes run one by
        one. Conv groups read and write the packed / channels-last layouts
        where that saves a pack, unpack or transpose (see _Laid)."""
        from .. import ops
        if not self._group_ready(g, values):
            return None
        head = g['head']
        op = self.stages[head.replace('.', '_')]
        xv = values.get(self._node_args[head][0])
        if g['kind'] == 'linear':
            return ops.linear(self._std(xv), op.weight, op.bias, act=g['act'])
        if g['kind'] == 'chain':
            return self._run_chain(g, xv)
        if g['kind'] == 'attn_ln':
            ln = self.stages[g['ln'].replace('.', '_')]
            out_ln = (ln.weight, ln.bias, ln.eps)
            if isinstance(xv, _Laid) and xv.layout == ops.LAYOUT_PACKED and xv.t.dim() == 3:
                return _Laid(ops.attention_packed(op, xv.t, g['is_causal'], out_ln), ops.LAYOUT_PACKED)
            x = self._std(xv)
            return ops.attention(op, x, x, x, None, g['is_causal'], out_ln)
        bn_mod = self.stages[g['bn'].replace('.', '_')].op
        w, b, st, pd, dl = self._conv_params(op)
        rv = values.get(g['residual']) if g['residual'] is not None else None
        t = xv.t if isinstance(xv, _Laid) else xv
        scale, shift = self._folded_bn(bn_mod, t.dtype)
        kw = dict(scale=scale, shift=shift, act=g['act'], residual_first=g['residual_first'])
        in_l = xv.layout if isinstance(xv, _Laid) else ops.LAYOUT_NFIRST
        res_l = rv.layout if isinstance(rv, _Laid) else ops.LAYOUT_NFIRST
        res_t = rv.t if isinstance(rv, _Laid) else rv
        # Output layout: packed when this group produces the model output,
        # channels-last when the only consumer is a fused conv group that can
        # read it (checked for its geometry), else N-first.
        out_l = ops.LAYOUT_NFIRST
        tail = g['nodes'][-1]
        nxt = self._next_conv_group(g)
        if tail == self._output_name and self._fusion.get('consumers', {}).get(tail) == ['<output>']:
            out_l = ops.LAYOUT_PACKED
        elif nxt is not None and self._group_ready(nxt, {**values, self._node_args[nxt['head']][0]: t}) \
                and self._clast_ok(nxt, op, t, in_l, w, st, pd, dl):
            # (the next group's readiness is judged with this group's output
            # standing in for its input; its residual must already exist)
            out_l = ops.LAYOUT_CLAST
        tries = [(in_l, out_l, res_l)]
        if out_l != ops.LAYOUT_NFIRST:
            tries.append((in_l, ops.LAYOUT_NFIRST, res_l))
        for il, ol, rl in tries:
            y = ops.conv_nd(t, w, b, op.n, st, pd, dl, residual=res_t, in_layout=il, out_layout=ol,
                            res_layout=rl, **kw)
            if y is not None:
                return _Laid(y, ol) if ol != ops.LAYOUT_NFIRST else y
        # Fall back to N-first tensors everywhere.
        xs = self._std(xv)
        res = self._std(rv) if rv is not None else None
        y = ops.conv_nd(xs, w, b, op.n, st, pd, dl, residual=res, **kw)
        if res is not None and y.shape != res.shape:
            return None
        return y

    def _folded_bn(self, bn_mod: nn.Module, dtype: torch.dtype):
        """The eval-mode BatchNorm as (scale, shift) in `dtype`, kept from one
        forward to the next (folding it costs about six small device
        launches per conv group). The entry is keyed on the module's four
        tensors (identity, storage, version) and eps
        (``wide_compiler._derived``), so replacing a tensor or changing it
        in place (``copy_``, an optimizer step, ``load_state_dict``,
        training-mode statistics) recomputes it; during CUDA-graph capture
        the fold is recorded into the graph, so replays fold the live
        tensors. In-place writes through ``.data`` leave the version
        unchanged: call ``invalidate_caches()`` after them."""
        tensors = (bn_mod.running_mean, bn_mod.running_var, bn_mod.weight, bn_mod.bias)

        def fold():
            scale, shift = _bn_fold(bn_mod)
            return scale.to(dtype), shift.to(dtype)

        return _derived.cached(bn_mod, ('bn_fold', dtype), tensors, fold, extra=float(bn_mod.eps))

    def invalidate_caches(self) -> None:
        """Drops every tensor derived from the parameters (folded BatchNorm,
        repacked conv weights, fused attention projections, LSTM blocks);
        the next forward rebuilds them. Needed only after in-place writes
        through ``.data`` (``p.data.copy_(...)``), which do not bump the
        version counters the caches are keyed on."""
        _derived.invalidate_caches(self)

    def _clast_ok(self, nxt: Dict[str, Any], op, t: Tensor, in_l: int, w, st, pd, dl) -> bool:
        """Whether the next conv group can read this group's output in the
        channels-last layout (its geometry, dtype and output layouts)."""
        import ctypes
        from .. import _native as N
        from .. import ops
        op2 = self.stages[nxt['head'].replace('.', '_')]
        w2, _, st2, pd2, dl2 = self._conv_params(op2)
        n = op.n
        if in_l == ops.LAYOUT_PACKED:
            batch, sp = t.shape[0], tuple(t.shape[2:])
        elif in_l == ops.LAYOUT_CLAST:
            batch, sp = t.shape[1], tuple(t.shape[2:-1])
        else:
            batch, sp = t.shape[1], tuple(t.shape[3:])
        nd = len(sp)
        if nd not in (1, 2) or w2.dim() != nd + 2:
            return False
        cout = w.shape[0] // n
        pad3 = lambda v, fill: (fill,) * (3 - nd) + tuple(v)
        ks, st_, pd_, dl_ = pad3(w.shape[2:], 1), pad3(st, 1), pad3(pd, 0), pad3(dl, 1)
        sp3 = pad3(sp, 1)
        osp = tuple((sp3[i] + 2 * pd_[i] - dl_[i] * (ks[i] - 1) - 1) // st_[i] + 1 for i in range(3))
        cout2 = w2.shape[0] // op2.n
        ks2, st2_, pd2_, dl2_ = pad3(w2.shape[2:], 1), pad3(st2, 1), pad3(pd2, 0), pad3(dl2, 1)
        osp2 = tuple((osp[i] + 2 * pd2_[i] - dl2_[i] * (ks2[i] - 1) - 1) // st2_[i] + 1 for i in range(3))
        if min(osp2) <= 0 or op2.n != n or w2.shape[1] != cout:
            return False
        geom = (ctypes.c_int64 * 22)(n, batch, cout, cout2, *osp, *ks2, *st2_, *pd2_, *dl2_, *osp2)
        has_res = 1 if nxt['residual'] is not None else 0
        return bool(N.lib().widek_conv_layouts_supported(geom, N.dtype_code(t), ops.LAYOUT_CLAST,
                                                         ops.LAYOUT_NFIRST, ops.LAYOUT_NFIRST, has_res))

    def _run_stages(self, x: Tensor, fused: bool = True) -> Any:
        if self._fusion is None:
            self._fusion = self._build_fusion_plan() if self.fuse else {'groups': {}, 'folded': set(),
                                                                        'consumers': {}, 'by_head': {}}
        groups, folded = (self._fusion['groups'], self._fusion['folded']) if fused else ({}, set())
        values: Dict[str, Any] = {self._input_name: x}
        for name in self._attr_names:
            buf = f"_attr_{name.replace('.', '_')}"
            if hasattr(self, buf):
                values[name] = getattr(self, buf)
        pending = []                      # folded nodes whose group fell back to node-by-node
        for name in self._execution_order:
            if name in self._attr_names or name not in self.stage_info:
                continue
            if name in folded:
                pending.append(name)
                continue
            if name in groups:
                y = self._run_group(groups[name], values)
                if y is not None:
                    values[name] = y
                    pending = [p for p in pending if p not in groups[name]['nodes']]
                    continue
                for p_name in groups[name]['nodes'][:-1]:
                    values[p_name] = self._run_node(p_name, values)
                pending = [p for p in pending if p not in groups[name]['nodes']]
            values[name] = self._run_node(name, values)
        return values[self._output_name]

    def _std(self, v: Any) -> Any:
        """The N-first tensor of a value (materialised once for _Laid)."""
        if not isinstance(v, _Laid):
            return v
        if v.std is None:
            from ..ops import LAYOUT_PACKED
            if v.layout != LAYOUT_PACKED:
                raise RuntimeError("TracedWideModel: internal channels-last value reached a non-conv consumer")
            v.std = self._unpack(v.t)
        return v.std

    def _packed_call(self, op: nn.Module, name: str, values: Dict[str, Any]) -> Any:
        """Runs a stage on the packed boundary layout when every tensor it
        reads is a packed value and the stage offers ``forward_packed``
        (norms, elementwise glue, recurrent and attention layers): the result
        stays packed, so neither the unpack before it nor, at the graph's end,
        the pack after it is needed. None when the stage declines."""
        fp = getattr(op, 'forward_packed', None)
        if fp is None:
            return None
        from ..ops import LAYOUT_PACKED

        def resolve(a):
            v = values[a] if isinstance(a, str) and a in values else a
            if isinstance(v, _Laid):
                return v.t if v.layout == LAYOUT_PACKED else _Decline
            if isinstance(v, (Tensor, tuple, list, dict)):
                return _Decline
            return v
        args = [resolve(a) for a in self._node_args[name]]
        kwargs = {k: resolve(v) for k, v in self._node_kwargs.get(name, {}).items()}
        if any(a is _Decline for a in args) or any(v is _Decline for v in kwargs.values()):
            return None
        if not any(isinstance(a, Tensor) for a in args):
            return None
        out = fp(*args, **kwargs)
        if out is None:
            return None
        if isinstance(out, tuple):
            return (_Laid(out[0], LAYOUT_PACKED),) + tuple(out[1:])
        return _Laid(out, LAYOUT_PACKED)

    def _run_node(self, name: str, values: Dict[str, Any]) -> Any:
        op = self.stages[name.replace('.', '_')]
        packed = self._packed_call(op, name, values)
        if packed is not None:
            return packed
        args = [self._std(values[a]) if isinstance(a, str) and a in values else a for a in self._node_args[name]]
        kwargs = {k: (self._std(values[v]) if isinstance(v, str) and v in values else v)
                  for k, v in self._node_kwargs.get(name, {}).items()}
        return op(*args, **kwargs)

    def _needs_grad(self, x: Tensor) -> bool:
        """Autograd wants this call's result: the fused group kernels have no
        gradient formulation, so such a call runs node by node, each wide op
        differentiable on its own."""
        if not torch.is_grad_enabled():
            return False
        return x.requires_grad or any(p.requires_grad for p in self.parameters())

    def forward(self, x: Tensor) -> Tensor:
        from ..ops import LAYOUT_PACKED
        # Under autograd, and while dynamo traces (torch.compile), the stages
        # run one by one on the differentiable / torch.library operators.
        if self._needs_grad(x) or torch.compiler.is_compiling():
            out = self._run_stages(self._unpack(x), fused=False)
            if isinstance(out, tuple):
                out = out[0]
            return self._pack(self._std(out))
        if self.fuse and x.is_cuda:
            b, nc = x.shape[0], x.shape[1]
            if nc % self.n != 0:
                raise ValueError(f"input dim 1 ({nc}) is not a multiple of N={self.n}")
            out = self._run_stages(_Laid(x, LAYOUT_PACKED))
        else:
            out = self._run_stages(self._unpack(x))
        if isinstance(out, tuple):
            out = out[0]
        if isinstance(out, _Laid):
            if out.layout == LAYOUT_PACKED:
                return out.t           # the last fused conv wrote the packed output
            out = self._std(out)
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
