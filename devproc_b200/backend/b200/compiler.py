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
from ..host_ops import split_host_ops
from .host_program import HostDeviceProgram
from .lowering import lower
from .program import B200CompiledProgram, ProgramSpec
from .rebatch import batch_factors, rebatch


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
        split = split_host_ops(ir_function)
        if split is not None:  # tokenizer / string / dict ops run on the host around one device plan
            prologue, sub, epilogue, dev_in, dev_out = split
            device = self.compile(sub, constants) if sub.block.ops else None
            return HostDeviceProgram.from_split(ir_function, prologue, device, epilogue, dev_in, dev_out)
        consts = dict(getattr(ir_function, "constants", {}) or {})
        consts.update(constants or {})
        low = lower(ir_function, const_names=consts.keys(), const_tensors=consts)
        consts.update(low.extra_consts)
        spec = ProgramSpec.from_lowered(low)
        prog = B200CompiledProgram(spec, consts, self.device_id, ir_function, self.use_graph)
        chunk = stream_chunk(ir_function, low, consts)
        if chunk is not None:
            sub_fn = rebatch(ir_function, chunk, consts.keys())
            sub = lower(sub_fn, const_names=consts.keys(), const_tensors=consts)
            consts.update(sub.extra_consts)
            prog.set_stream(chunk, ProgramSpec.from_lowered(sub))
        return prog


# Streaming a program in chunks pays when its run is dominated by moving
# host data: only memory-bound records (no GEMM or attention), and enough
# input bytes that each chunk's copy is still long next to a launch.
_STREAM_MIN_BYTES = 16 << 20
_STREAM_MIN_CHUNK_BYTES = 4 << 20
_STREAM_MAX_CHUNKS = 16


def stream_chunk(fn: Function, low, consts) -> Optional[int]:
    """Chunk batch for overlapped host transfers, or None: the program must be
    batch-separable and memory-bound, with at least 16 MiB of input."""
    from ... import _native as N
    if any(r.kernel in (N.DP_K_GEMM, N.DP_K_ATTENTION) for r in low.records):
        return None
    B, _, _ = batch_factors(fn, consts.keys())
    if B is None:
        return None
    in_bytes = sum(b.nbytes for _, b in low.inputs)
    if in_bytes < _STREAM_MIN_BYTES:
        return None
    n = min(_STREAM_MAX_CHUNKS, B, in_bytes // _STREAM_MIN_CHUNK_BYTES)
    for chunk in range(-(-B // n), B):
        if B % chunk == 0:
            return chunk
    return None
