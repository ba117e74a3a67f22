"""DevProc on B200: the DevProc Python API over hand-written sm_100a kernels.

Same public surface as the reference package (src/devproc/__init__.py:1-177):
the IR classes, the ``@kernel`` DSL and its op functions, ``from_torch``,
``compile`` / ``save`` / ``load`` and ``Runtime``.  ``compile`` lowers the IR
to launch records over a compile-time arena and returns a program that runs
on the C-ABI library ``libdevproc_b200.so``; there is no other execution
path.  The reference's ``TritonCompiler`` / ``TritonCompiledProgram`` /
``TritonRuntime`` names remain importable as aliases of the B200 classes, and
``backend="triton"`` selects the B200 backend, so reference code runs
unchanged.
"""

from .ir.types import Type, TensorType, ScalarType, StringType, TokenizerType, DictType, ListType
from .ir.base import Value, Op
from .ir.function import Function, Block
from .ir.ops import OpBuilder
from .ir.verifier import IRVerifier
from .dsl.kernel import kernel, KernelTensor, parse_ir
from .dsl import ops as _ops
from .dsl.types import (String, Tensor, Float32, Float16, BFloat16, Int32, Int64, UInt8, Bool, Tokenizer,
                        TorchModel, KVCache, IRFunction)
from .ir.from_torch import from_export, from_torch
from .ir.export_importer import TorchExportImporter
from .runtime import Runtime
from .backend.base import Backend, CompiledProgram, BackendError, UnsupportedOpError, CompilationError
from .backend.b200 import B200Compiler, B200CompiledProgram
from ._native import DevProcError

__version__ = "0.1.0"

load_image = _ops.load_image
input = _ops.input
resize = _ops.resize
to = _ops.to
normalize = _ops.normalize
transpose = _ops.transpose
reshape = _ops.reshape
matmul = _ops.matmul
linear = _ops.linear
relu = _ops.relu
sigmoid = _ops.sigmoid
gelu = _ops.gelu
tanh = _ops.tanh
silu = _ops.silu
exp = _ops.exp
softmax = _ops.softmax
add = _ops.add
sub = _ops.sub
mul = _ops.mul
div = _ops.div
argmax = _ops.argmax
sum = _ops.sum
max = _ops.max
mean = _ops.mean
layer_norm = _ops.layer_norm
rms_norm = _ops.rms_norm
embedding = _ops.embedding
sdpa = _ops.sdpa
slice = _ops.slice
cat = _ops.cat
rope = _ops.rope
load_vla_module = _ops.load_vla_module
# For torch modules: a rotary embedding that capture keeps as one op.
from .torch_ops import rope as torch_rope, rope_tables  # noqa: E402

# Reference names (src/devproc/__init__.py:46-47) kept as aliases of the only backend.
TritonCompiler = B200Compiler
TritonCompiledProgram = B200CompiledProgram


class TritonRuntime:
    """Reference-compatible runtime wrapper (compiler.py:539-633): ``execute(program, **inputs)``."""

    def __init__(self, device_id: int = 0):
        self.device_id = device_id

    def execute(self, program, **inputs):
        return program.run(**inputs)


_BACKENDS = ("b200", "triton", "cuda")


def compile(target, *example_inputs, backend: str = "b200", **kwargs):
    """Compile a ``@kernel`` function, an IR Function or a torch module.

    ``target`` may be an IR ``Function``; a ``@kernel`` wrapper or plain
    function (called with ``example_inputs`` to build the IR, as in the
    reference, __init__.py:55-85); a ``torch.nn.Module``, captured with
    Dynamo (``method="dynamo"``) or ``torch.export`` (``method="export"``);
    or a ``torch.export.ExportedProgram``.  ``kwargs``: ``device_id``,
    ``use_graph``, ``constants`` (name → tensor bound once, e.g. weights).
    """
    if backend not in _BACKENDS:
        raise ValueError(f"Unknown backend: {backend}")
    constants = kwargs.pop("constants", None)
    method = kwargs.pop("method", "dynamo")
    if hasattr(target, "ir_function"):
        fn = target.ir_function
    elif isinstance(target, Function):
        fn = target
    elif isinstance(target, __import__("torch").export.ExportedProgram):
        fn = from_export(target, backend="ir")
    elif isinstance(target, __import__("torch").nn.Module):
        fn = from_torch(target, *example_inputs, backend="ir", method=method)
    else:
        fn = target(*example_inputs)
    return B200Compiler(**kwargs).compile(fn, constants=constants)


from .sharded import ShardedRuntime, shard_batch, shard_range  # noqa: E402


def save(compiled_program, path: str) -> None:
    """Write ``path`` (plan), ``path.meta.json`` and, with constants, ``path.weights``."""
    compiled_program.export(path)


def load(path: str, device_id: int = 0):
    """Load a program written by ``save``."""
    return B200CompiledProgram.load(path, device_id=device_id)


__all__ = [
    "Type", "TensorType", "ScalarType", "StringType", "TokenizerType", "DictType", "ListType",
    "Value", "Op", "Function", "Block", "OpBuilder", "IRVerifier",
    "kernel", "KernelTensor", "parse_ir",
    "String", "Tensor", "Float32", "Float16", "BFloat16", "Int32", "Int64", "UInt8", "Bool", "Tokenizer",
    "TorchModel", "KVCache", "IRFunction",
    "load_image", "input", "resize", "to", "normalize", "transpose", "reshape", "matmul", "linear", "relu",
    "sigmoid", "gelu", "tanh", "silu", "exp", "softmax", "add", "sub", "mul", "div", "argmax", "sum", "max",
    "mean", "layer_norm", "rms_norm", "embedding", "load_vla_module",
    "Backend", "CompiledProgram", "BackendError", "UnsupportedOpError", "CompilationError",
    "B200Compiler", "B200CompiledProgram", "TritonCompiler", "TritonCompiledProgram", "TritonRuntime",
    "DevProcError", "Runtime", "compile", "save", "load", "from_torch", "from_export", "TorchExportImporter",
    "ShardedRuntime", "shard_batch", "shard_range",
]
