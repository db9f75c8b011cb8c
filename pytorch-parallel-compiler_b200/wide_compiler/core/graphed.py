"""GraphedWideModel: the CUDA-graph executor behind ``compile(..., compile_model=True)``.

The reference hands its TracedWideModel to ``torch.compile`` (default mode
'reduce-overhead', i.e. Inductor plus CUDA graphs; reference
wide_compiler/api.py:137-147 and core/config.py:46-49). Here the stages
already run as sm_100a kernels, so what is left to remove is the host work
per call: Python dispatch of every stage and one kernel launch per fused
group. This executor records the whole forward of a TracedWideModel into
one CUDA graph per input signature and replays it:

* A signature is the input's device pointer, shape, strides, dtype and
  device and the model's fusion switch and mode; a recorded graph is
  replayed only while the model's parameters and buffers still live where
  it read them (a ``.to()`` of the model records anew; after replacing a
  Parameter object itself call ``reset()``). A serving loop that reuses its
  input buffers replays without any copy; a new buffer records a new graph.
  At most ``max_graphs`` graphs are kept (least recently used dropped).
* Recording happens on the first call with a signature: two eager warm-up
  runs on a side stream (they build the fusion plan and set the kernels'
  shared-memory limits), then capture. Later calls replay.
* Tensors derived from the parameters (folded BatchNorm, repacked conv
  weights, the fused [q; kv] projection, LSTM diagonal blocks) are rebuilt
  inside the graph, so a replay always reads the live parameters: in-place
  updates (``mul_``, an optimizer step, ``load_state_dict``, and writes
  through ``.data``) are seen by the next replay without recording again.
* Like torch.compile's 'reduce-overhead' mode, a call returns the graph's
  static output tensor, which the next replay of the same graph
  overwrites; ``clone()`` it to keep it.
* Inputs larger than ``max_input_bytes`` (default 32 MiB) run eagerly:
  at that size the kernels, not the launches, set the time. CPU inputs also
  run eagerly (and fail loudly in the kernels, as the eager model does), and
  so do calls whose result autograd needs (grad mode on and a parameter or
  the input requiring grad): replays are for inference (``torch.no_grad()``
  / ``torch.inference_mode()``).
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Any, Optional

import torch
import torch.nn as nn
from torch import Tensor

from .. import _native


class _Recorded:
    __slots__ = ('graph', 'output', 'tensors', 'ptrs', 'launches')

    def __init__(self, graph, output, tensors, launches):
        self.graph, self.output, self.tensors = graph, output, tensors
        self.ptrs = tuple(t.data_ptr() for t in tensors)
        self.launches = launches            # library kernels one replay runs

    def current(self) -> bool:
        """The parameters and buffers still live where the graph reads them."""
        for t, p in zip(self.tensors, self.ptrs):
            if t.data_ptr() != p:
                return False
        return True


class GraphedWideModel(nn.Module):
    """Wraps a TracedWideModel (as ``_orig_mod``, the attribute name
    torch.compile's wrapper uses) and replays its forward from CUDA graphs."""

    def __init__(self, model: nn.Module, max_graphs: int = 8, max_input_bytes: int = 32 << 20):
        super().__init__()
        self._orig_mod = model
        self.max_graphs = max_graphs
        self.max_input_bytes = max_input_bytes
        self._graphs: 'OrderedDict[Any, Optional[_Recorded]]' = OrderedDict()

    def __getattr__(self, name: str):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self._modules['_orig_mod'], name)

    def _signature(self, x: Tensor):
        m = self._orig_mod
        return (x.data_ptr(), x.shape, x.stride(), x.dtype, x.device, getattr(m, 'fuse', None), m.training)

    def _record(self, x: Tensor) -> _Recorded:
        m = self._orig_mod
        side = torch.cuda.Stream(x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            for _ in range(2):
                m(x)
        torch.cuda.current_stream(x.device).wait_stream(side)
        # each graph keeps a private memory pool, so graphs recorded for
        # different inputs may also be replayed on different streams
        g = torch.cuda.CUDAGraph()
        n0 = _native.launch_count()
        with torch.cuda.graph(g):
            out = m(x)
        return _Recorded(g, out, list(m.parameters()) + list(m.buffers()), _native.launch_count() - n0)

    def reset(self) -> None:
        """Drops every recorded graph (they are recorded again on demand)."""
        self._graphs.clear()

    def forward(self, x: Tensor) -> Tensor:
        if not isinstance(x, Tensor) or not x.is_cuda or x.numel() * x.element_size() > self.max_input_bytes:
            return self._orig_mod(x)
        if torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in self.parameters())):
            return self._orig_mod(x)           # autograd wants the result: no graph replay
        key = self._signature(x)
        rec = self._graphs.get(key)
        if rec is None or not rec.current():
            if rec is None and len(self._graphs) >= self.max_graphs:
                self._graphs.popitem(last=False)
            rec = self._record(x)
            self._graphs[key] = rec
        self._graphs.move_to_end(key)
        rec.graph.replay()
        _native.note_replayed_launches(rec.launches)
        return rec.output

    def extra_repr(self) -> str:
        return f"graphs={len(self._graphs)}, max_graphs={self.max_graphs}"
