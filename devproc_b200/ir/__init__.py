"""DevProc IR: types, values/ops, functions, builders, verifier, FX frontend."""

from .types import Type, TensorType, ScalarType, StringType, TokenizerType, DictType, ListType
from .base import Value, Op
from .function import Function, Block
from .ops import OpBuilder
from .verifier import IRVerifier
from .from_torch import from_torch, DevProcDynamoBackend, DevProcCompiledProgram
from .fx_converter import FXToIRConverter
from .fx_op_map import get_fx_op_map

__all__ = ["Type", "TensorType", "ScalarType", "StringType", "TokenizerType", "DictType", "ListType",
           "Value", "Op", "Function", "Block", "OpBuilder", "IRVerifier", "from_torch",
           "DevProcDynamoBackend", "DevProcCompiledProgram", "FXToIRConverter", "get_fx_op_map"]
