"""sm_100a backend: lowering, compiled program and compiler."""

from .compiler import B200Compiler
from .program import B200CompiledProgram, ProgramSpec

__all__ = ["B200Compiler", "B200CompiledProgram", "ProgramSpec"]
