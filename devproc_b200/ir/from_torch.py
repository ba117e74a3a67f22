"""Torch frontend: capture a module or function with Dynamo and convert to IR.

Reference: src/devproc/ir/from_torch.py:21-159.  ``from_torch(target,
*example_inputs, backend="ir")`` returns the IR Function;
``backend="devproc"`` compiles it with the B200 backend and returns a
callable program, with the module's parameters uploaded once as constants.
``DevProcDynamoBackend`` can also be handed to ``torch.compile`` directly.
"""

from typing import Any, Callable, Optional, Tuple, Union

import torch

from .function import Function
from .export_importer import TorchExportImporter, export_module
from .fx_converter import FXToIRConverter


class DevProcDynamoBackend:
    """A ``torch.compile`` backend that compiles the captured graph with the B200 backend."""

    def __init__(self, device_id: int = 0):
        self.device_id = device_id
        self.graph_module: Optional[torch.fx.GraphModule] = None
        self.ir_function: Optional[Function] = None
        self.example_inputs: Optional[Tuple[Any, ...]] = None
        self.program = None

    def __call__(self, gm: torch.fx.GraphModule, example_inputs):
        from ..backend.b200 import B200Compiler
        self.graph_module = gm
        self.example_inputs = tuple(example_inputs)
        self.ir_function = FXToIRConverter().convert(gm, self.example_inputs)
        self.program = B200Compiler(self.device_id).compile(self.ir_function)
        runtime_inputs = [i for i, v in enumerate(self.ir_function.inputs)
                          if v.name not in self.ir_function.constants]
        prog = self.program

        def run(*args):
            outs = prog.run(*[args[i] for i in runtime_inputs], to_cpu=False)
            return tuple(o.clone() for o in outs)

        return run


class DevProcCompiledProgram:
    """Callable wrapper of a compiled program (reference from_torch.py:72-83)."""

    def __init__(self, compiled_program):
        self._compiled = compiled_program

    def __call__(self, *args, **kwargs):
        return self._compiled.run(*args, **kwargs)

    def run(self, *args, **kwargs):
        return self._compiled.run(*args, **kwargs)

    @property
    def program(self):
        return self._compiled


def capture(target: Union[torch.nn.Module, Callable], *example_inputs) -> Tuple[torch.fx.GraphModule, tuple]:
    """Dynamo-capture ``target`` once; returns (graph module, real example inputs incl. lifted params)."""
    captured = {}

    def backend(gm, ex):
        if "gm" in captured:
            raise ValueError("the model breaks into several graphs; DevProc needs one static graph")
        captured["gm"], captured["ex"] = gm, tuple(ex)
        return gm.forward

    torch._dynamo.reset()
    compiled = torch.compile(target, backend=backend, fullgraph=True, dynamic=False)
    with torch.no_grad():
        compiled(*example_inputs)
    torch._dynamo.reset()
    if "gm" not in captured:
        raise ValueError("Failed to capture FX graph")
    return captured["gm"], captured["ex"]


def from_torch(target: Union[torch.nn.Module, Callable], *example_inputs: Any, backend: str = "devproc",
               device_id: int = 0, method: str = "dynamo"):
    """Convert ``target`` to IR (``backend="ir"``) or to a compiled program (``"devproc"``).

    ``method="dynamo"`` captures with ``torch.compile`` (the reference's FX
    path); ``method="export"`` goes through ``torch.export.export`` and the
    ATen importer.  ``target`` may also be an ``ExportedProgram``."""
    if backend not in ("ir", "devproc"):
        raise ValueError(f"Unknown backend: {backend}")
    if method not in ("dynamo", "export"):
        raise ValueError(f"Unknown capture method: {method}")
    if isinstance(target, torch.export.ExportedProgram):
        fn = TorchExportImporter().import_program(target)
    elif method == "export":
        fn = TorchExportImporter().import_program(export_module(target, *example_inputs))
    else:
        gm, ex = capture(target, *example_inputs)
        fn = FXToIRConverter().convert(gm, ex)
    if backend == "ir":
        return fn
    from ..backend.b200 import B200Compiler
    return DevProcCompiledProgram(B200Compiler(device_id).compile(fn))


def from_export(ep: "torch.export.ExportedProgram", backend: str = "devproc", device_id: int = 0):
    """IR (``backend="ir"``) or compiled program of a ``torch.export`` result."""
    return from_torch(ep, backend=backend, device_id=device_id)
