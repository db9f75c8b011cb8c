"""Imports the reference package (WideCompiler, pure Python) from its source
tree under the alias ``ref_wide_compiler``, so that it can live in the same
process as this repository's ``wide_compiler``. Used only to generate and
cross-check golden fixtures on a machine that has the reference checkout."""
from __future__ import annotations

import importlib.util
import os
import sys

# The reference checkout's root directory (the one holding wide_compiler/),
# given by the environment; there is no built-in default.
DEFAULT_ROOT = os.environ.get("WIDE_REFERENCE_ROOT", "")
ALIAS = "ref_wide_compiler"


def available(root: str = DEFAULT_ROOT) -> bool:
    return bool(root) and os.path.exists(os.path.join(root, "wide_compiler", "__init__.py"))


def load(root: str = DEFAULT_ROOT):
    if ALIAS in sys.modules:
        return sys.modules[ALIAS]
    pkg_dir = os.path.join(root, "wide_compiler")
    spec = importlib.util.spec_from_file_location(ALIAS, os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[ALIAS] = mod
    spec.loader.exec_module(mod)
    return mod
