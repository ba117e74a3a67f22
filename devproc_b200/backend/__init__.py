"""Backend plugin contract and the B200 backend."""

from .base import Backend, BackendError, CompilationError, CompiledProgram, UnsupportedOpError

__all__ = ["Backend", "CompiledProgram", "BackendError", "UnsupportedOpError", "CompilationError"]
