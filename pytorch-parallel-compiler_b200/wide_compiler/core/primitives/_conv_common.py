"""Shared helpers for the wide convolutions (1-D, 2-D, 3-D)."""
from __future__ import annotations

from typing import Sequence, Tuple, Union

IntOrTuple = Union[int, Sequence[int]]


def ntuple(v: IntOrTuple, n: int) -> Tuple[int, ...]:
    if isinstance(v, (tuple, list)):
        if len(v) == 1:
            return tuple(int(v[0]) for _ in range(n))
        if len(v) != n:
            raise ValueError(f"expected {n} values, got {tuple(v)}")
        return tuple(int(e) for e in v)
    return tuple(int(v) for _ in range(n))


def check_padding(padding) -> None:
    if isinstance(padding, str):
        raise ValueError("string padding modes ('same'/'valid') are not supported by the wide convolutions; "
                         "pass explicit integers")
