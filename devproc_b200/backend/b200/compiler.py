"""The B200 backend: IR Function → B200CompiledProgram.

Drop-in for TritonCompiler (src/devproc/backend/triton/compiler.py:452-536):
same constructor argument (``device_id``), same ``name`` / ``is_available`` /
``compile`` contract.  Compilation is host-only — it verifies the IR, lowers
it to launch records and plans the arena; no GPU is touched until the first
``run`` (the reference launched every template once at compile time,
aot.py:166-180).
"""

from typing import Dict, Optional

import torch

from ...ir.function import Function
from ...ir.verifier import IRVerifier
from ..base import Backend, CompilationError
from .lowering import lower
from .program import B200CompiledProgram, ProgramSpec


class B200Compiler(Backend):
    def __init__(self, device_id: int = 0, use_graph: bool = True, verify: bool = True):
        self.device_id = device_id
        self.use_graph = use_graph
        self.verify = verify

    @property
    def name(self) -> str:
        return "b200"

    def is_available(self) -> bool:
        if not torch.cuda.is_available():
            return False
        major, minor = torch.cuda.get_device_capability(self.device_id)
        return (major, minor) == (10, 0)

    def compile(self, ir_function: Function,
                constants: Optional[Dict[str, torch.Tensor]] = None) -> B200CompiledProgram:
        if not isinstance(ir_function, Function):
            raise TypeError(f"expected an IR Function, got {type(ir_function).__name__}")
        if self.verify:
            v = IRVerifier(ir_function)
            if not v.verify():
                raise CompilationError("IR verification failed: " + "; ".join(v.get_errors()))
        consts = dict(getattr(ir_function, "constants", {}) or {})
        consts.update(constants or {})
        low = lower(ir_function, const_names=consts.keys(), const_tensors=consts)
        consts.update(low.extra_consts)
        spec = ProgramSpec.from_lowered(low)
        return B200CompiledProgram(spec, consts, self.device_id, ir_function, self.use_graph)
