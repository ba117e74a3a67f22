"""``import devproc`` → this package's B200 implementation (drop-in name).

Code written against the reference (``import devproc``,
``from devproc.ir.verifier import IRVerifier``, ``from devproc.backend.base
import Backend`` …) resolves to ``devproc_b200`` and its submodules.
"""

import importlib
import sys

import devproc_b200 as _impl
from devproc_b200 import *  # noqa: F401,F403
from devproc_b200 import __all__, __version__  # noqa: F401

_SUBMODULES = [
    "ir", "ir.types", "ir.base", "ir.function", "ir.ops", "ir.verifier", "ir.from_torch", "ir.fx_converter",
    "ir.fx_op_map", "dsl", "dsl.kernel", "dsl.ops", "dsl.types", "runtime", "backend", "backend.base",
    "backend.b200", "backend.b200.compiler", "backend.b200.program", "backend.b200.lowering", "sharded",
]
for _name in _SUBMODULES:
    sys.modules[f"{__name__}.{_name}"] = importlib.import_module(f"devproc_b200.{_name}")
ir = _impl.ir
dsl = _impl.dsl
runtime = _impl.runtime
backend = _impl.backend
