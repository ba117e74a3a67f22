"""Backend plugin contract (reference: src/devproc/backend/base.py:12-140).

``Backend`` compiles an IR Function into a ``CompiledProgram``; a compiled
program runs with keyword inputs named after the IR inputs, exports to a path
and loads back.  The error classes keep the reference's names.
"""

from abc import ABC, abstractmethod
from typing import Any, Dict, List

from ..ir.function import Function


class Backend(ABC):
    @property
    @abstractmethod
    def name(self) -> str:
        """Backend name."""

    @abstractmethod
    def compile(self, ir_function: Function) -> "CompiledProgram":
        """Compile ``ir_function``."""

    @abstractmethod
    def is_available(self) -> bool:
        """True when the backend can run on this machine."""


class CompiledProgram(ABC):
    @abstractmethod
    def run(self, **kwargs) -> List[Any]:
        """Execute; inputs by IR input name; returns the output tensors."""

    @abstractmethod
    def export(self, path: str) -> None:
        """Write the program to ``path`` (plus ``path + '.meta.json'``)."""

    @staticmethod
    @abstractmethod
    def load(path: str, device_id: int = 0) -> "CompiledProgram":
        """Read a program written by ``export``."""


class LoweringContext:
    """Name → tensor table used while lowering (reference base.py:82-122)."""

    def __init__(self, backend: Backend):
        self.backend = backend
        self.tensor_map: Dict[str, Any] = {}
        self.kernel_cache: Dict[str, Any] = {}

    def allocate_tensor(self, name: str, shape: tuple, dtype: str, device: str) -> Any:
        raise NotImplementedError

    def get_tensor(self, name: str) -> Any:
        return self.tensor_map.get(name)

    def set_tensor(self, name: str, tensor: Any) -> None:
        self.tensor_map[name] = tensor


class BackendError(Exception):
    """Base class of backend errors."""


class UnsupportedOpError(BackendError):
    def __init__(self, op_name: str):
        self.op_name = op_name
        super().__init__(f"Operation '{op_name}' is not supported by this backend")


class CompilationError(BackendError):
    """Raised when an IR function cannot be lowered."""
