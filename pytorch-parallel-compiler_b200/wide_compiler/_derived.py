"""Caches of tensors derived from parameters (repacked or concatenated weights).

Several kernels read a re-laid-out copy of a parameter instead of the
parameter itself: the conv weight in [rows, taps, cin] order, the fused
[q; kv] attention projection, the dense diagonal blocks of WideLSTM's
block-diagonal matrices, the folded eval BatchNorm (scale, shift). Building
them costs launches, so they are kept from one forward to the next.

Validity. An entry is keyed on every source tensor's identity, storage
pointer, version counter, dtype and shape, so it is rebuilt after
``copy_`` / ``mul_`` / an optimizer step / ``load_state_dict`` (all bump the
version) and after ``p.data = other`` (new storage). Writes made through
``p.data`` in place (``p.data.copy_(...)``, common in EMA and weight-sync
code) do not bump the version counter and cannot be seen from the host;
after such writes call :func:`invalidate_caches` on the module (also
``TracedWideModel.invalidate_caches()`` and the compiled model's method of
the same name).

CUDA graphs. While a CUDA graph is being captured nothing is cached: the
derived tensor is built inside the graph from the live parameters, so every
replay re-derives it and a recorded graph can never read a stale copy (this
also holds for in-place ``.data`` writes). Inference-mode tensors have no
version counter; their derived tensors are built on every call.
"""
from __future__ import annotations

from typing import Any, Callable, Optional, Sequence

import torch
from torch import Tensor

_SLOTS_ATTR = '_widek_derived'


def _capturing() -> bool:
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


def _key(sources: Sequence[Optional[Tensor]], extra: Any):
    parts = []
    for t in sources:
        if t is None:
            parts.append(None)
        else:
            parts.append((id(t), t.data_ptr(), t._version, t.dtype, tuple(t.shape), t.device))
    return (tuple(parts), extra)


def cached(owner: Any, slot: str, sources: Sequence[Optional[Tensor]], build: Callable[[], Any],
           extra: Any = None) -> Any:
    """``build()`` memoised on ``owner`` under ``slot``, valid while every
    tensor in ``sources`` keeps its identity, storage, version, dtype and
    shape (and ``extra`` is unchanged). Built afresh, and not stored, during
    CUDA-graph capture and for tensors without a version counter."""
    if _capturing():
        return build()
    try:
        key = _key(sources, extra)
    except RuntimeError:                 # inference tensors: no version counter
        return build()
    store = owner.__dict__.setdefault(_SLOTS_ATTR, {})
    hit = store.get(slot)
    if hit is not None and hit[0] == key:
        return hit[1]
    value = build()
    # The sources are held so that their ids cannot be reused by new tensors
    # while the entry lives (the owner itself is not: the entry dies with it).
    store[slot] = (key, value, tuple(t for t in sources if t is not owner))
    return value


def _clear(obj: Any) -> None:
    d = getattr(obj, '__dict__', None)
    if d is not None and _SLOTS_ATTR in d:
        d[_SLOTS_ATTR].clear()


def invalidate_caches(module: torch.nn.Module) -> None:
    """Drops every derived tensor held by ``module``, its submodules and
    their parameters and buffers; the next forward rebuilds them. Needed
    only after in-place writes through ``.data``, which leave the version
    counter unchanged."""
    for m in module.modules():
        _clear(m)
        for t in list(m.parameters(recurse=False)) + list(m.buffers(recurse=False)):
            _clear(t)
