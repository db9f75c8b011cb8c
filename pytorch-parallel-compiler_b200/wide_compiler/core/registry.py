"""Public registry of wide primitives: module type name -> ``from_modules``.

Same API as the reference (wide_compiler/core/registry.py:20-232): a
``WideRegistry`` class, a process-wide instance with module-level helpers,
and auto-registration of the 14 built-in primitives on import. As in the
reference, ``TracedWideModel`` builds stages from its own ``WIDE_BUILDERS``
table (traced_wide.py); both tables name the same kernel-backed classes.
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional, Type

import torch.nn as nn

Builder = Callable[[List[nn.Module]], nn.Module]


class WideRegistry:
    """Maps a module type name (e.g. ``'Linear'``) to its Wide class."""

    def __init__(self):
        self._builders: Dict[str, Builder] = {}
        self._classes: Dict[str, Type[nn.Module]] = {}

    def register(self, module_type: str, wide_class: Optional[Type[nn.Module]] = None):
        """Registers ``wide_class`` (direct call) or returns a class decorator.

        Raises TypeError if the class has no ``from_modules``.
        """
        def add(cls: Type[nn.Module]) -> Type[nn.Module]:
            if not hasattr(cls, 'from_modules'):
                raise TypeError(
                    f"{cls.__name__} must implement classmethod from_modules(modules: List[nn.Module])")
            self._classes[module_type] = cls
            self._builders[module_type] = cls.from_modules
            return cls

        if wide_class is not None:
            return add(wide_class)
        return add

    def unregister(self, module_type: str) -> None:
        self._builders.pop(module_type, None)
        self._classes.pop(module_type, None)

    def get_builder(self, module_type: str) -> Optional[Builder]:
        return self._builders.get(module_type)

    def get_class(self, module_type: str) -> Optional[Type[nn.Module]]:
        return self._classes.get(module_type)

    def has(self, module_type: str) -> bool:
        return module_type in self._builders

    def build(self, modules: List[nn.Module]) -> Optional[nn.Module]:
        """Builds the wide module for ``modules`` (None if unregistered/empty)."""
        if not modules:
            return None
        builder = self._builders.get(type(modules[0]).__name__)
        return builder(modules) if builder is not None else None

    def list_registered(self) -> List[str]:
        return list(self._builders)

    def __contains__(self, module_type: str) -> bool:
        return self.has(module_type)

    def __repr__(self) -> str:
        return f"WideRegistry([{', '.join(sorted(self._builders))}])"


_global_registry = WideRegistry()


def get_registry() -> WideRegistry:
    return _global_registry


def register(module_type: str, wide_class: Optional[Type[nn.Module]] = None):
    return _global_registry.register(module_type, wide_class)


def unregister(module_type: str) -> None:
    _global_registry.unregister(module_type)


def get_builder(module_type: str) -> Optional[Builder]:
    return _global_registry.get_builder(module_type)


def build_wide(modules: List[nn.Module]) -> Optional[nn.Module]:
    return _global_registry.build(modules)


def list_registered() -> List[str]:
    return _global_registry.list_registered()


def auto_register_primitives() -> None:
    """Registers every built-in primitive under its torch.nn type name."""
    from . import primitives as P
    for name, cls in P.BUILTIN_PRIMITIVES.items():
        _global_registry.register(name, cls)


auto_register_primitives()

__all__ = ['WideRegistry', 'get_registry', 'register', 'unregister', 'get_builder', 'build_wide',
           'list_registered', 'auto_register_primitives']
