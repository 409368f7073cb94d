"""TEST INFRASTRUCTURE ONLY: modules of the reference's ``kernel_gen`` package, for CPU tests that
check this package against the reference's own code where a reference checkout is present.

Several of the reference's package ``__init__`` files import xdsl (absent here): importing
``kernel_gen.execute_engine.runtime_args`` normally runs ``kernel_gen/execute_engine/__init__.py``
-> ``compiler.py`` -> ``builtin_strategy`` -> ``kernel_gen.core.tools.dump_dir`` (xdsl), and
``kernel_gen.symbol_variable/__init__.py`` -> ``memory.py`` -> ``kernel_gen.core.contracts``
(xdsl). The modules the slot ABI, the strategy registry and the target registry live in need
none of that: ``runtime_args.py`` imports only ``kernel_gen.core.error`` and
``kernel_gen.symbol_variable.type``; ``strategy.py`` imports ``kernel_gen.core.error`` and
``kernel_gen.target.registry``. So the two packages are entered as bare package objects (their
``__path__`` only) and the modules are imported from the checkout unchanged.

The reference checkout is found as the oracle finds it (``oracle.reference_root()``:
$KG_REFERENCE_ROOT, else a checkout named ``reference`` beside this repository). Nothing on the
GPU box reads it: tests that need it skip when it is absent.
"""

from __future__ import annotations

import importlib
import sys
import types

import oracle

_BARE_PACKAGES = ("kernel_gen.execute_engine", "kernel_gen.symbol_variable")


def root():
    return oracle.reference_root()


def load(module: str):
    """The reference module `module` (e.g. "kernel_gen.execute_engine.runtime_args"), or None when
    no reference checkout is present."""
    ref = root()
    if ref is None:
        return None
    if str(ref) not in sys.path:
        sys.path.append(str(ref))
    for name in _BARE_PACKAGES:
        if name not in sys.modules:
            pkg = types.ModuleType(name)
            pkg.__path__ = [str(ref / name.replace(".", "/"))]
            sys.modules[name] = pkg
    return importlib.import_module(module)
