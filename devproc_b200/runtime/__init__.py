"""Runtime facade (reference: src/devproc/runtime/__init__.py:6-45).

``Runtime(compiled_or_path, device_id)`` wraps a compiled program, or loads
one from a path written by ``save``.  ``__call__`` and ``run`` both execute
it (the reference only had ``__call__``).
"""

from typing import Any, List, Union


class Runtime:
    def __init__(self, compiled_or_path: Union[Any, str], device_id: int = 0):
        if isinstance(compiled_or_path, str):
            from ..backend.b200.program import B200CompiledProgram
            self._compiled = B200CompiledProgram.load(compiled_or_path, device_id)
        else:
            self._compiled = compiled_or_path
        self._device_id = device_id

    def run(self, *args: Any, **kwargs: Any) -> List[Any]:
        return self._compiled.run(*args, **kwargs)

    def __call__(self, *args: Any, **kwargs: Any) -> List[Any]:
        return self._compiled.run(*args, **kwargs)

    @property
    def device_id(self) -> int:
        return self._device_id

    @property
    def program(self):
        return self._compiled


__all__ = ["Runtime"]
