"""Function and Block of the DevProc IR.

Reference: src/devproc/ir/function.py:9-143.  One block per function, inputs
are parameters (``input`` ops are not placed in the block), ``output`` is the
returned Value.  This build also accepts several returned values through
``outputs`` (``output`` stays the first one).
"""

import itertools
from typing import Dict, List, Optional

from .base import Op, Value


class Block:
    """Straight-line list of ops plus a name → Value table of their results."""

    def __init__(self):
        self._ops: List[Op] = []
        self._values: Dict[str, Value] = {}

    @property
    def ops(self) -> List[Op]:
        return self._ops

    @property
    def values(self) -> Dict[str, Value]:
        return self._values

    def add_op(self, op: Op) -> None:
        self._ops.append(op)
        for out in op.outputs:
            self._values[out.name] = out

    def get_value(self, name: str) -> Optional[Value]:
        return self._values.get(name)

    def __repr__(self) -> str:
        return "\n".join(["Block {"] + [f"  {op}" for op in self._ops] + ["}"])


class Function:
    """A named IR function: ordered inputs, one block, returned value(s)."""

    _names = itertools.count(1)

    def __init__(self, name: str):
        self._name = name
        self._inputs: List[Value] = []
        self._outputs: List[Value] = []
        self._block = Block()

    @property
    def name(self) -> str:
        return self._name

    @property
    def inputs(self) -> List[Value]:
        return self._inputs

    @property
    def output(self) -> Optional[Value]:
        return self._outputs[0] if self._outputs else None

    @output.setter
    def output(self, value: Optional[Value]) -> None:
        self._outputs = [] if value is None else [value]

    @property
    def outputs(self) -> List[Value]:
        return list(self._outputs)

    @outputs.setter
    def outputs(self, values: List[Value]) -> None:
        self._outputs = list(values)

    @property
    def block(self) -> Block:
        return self._block

    def add_input(self, value: Value) -> None:
        self._inputs.append(value)

    def add_op(self, op: Op) -> None:
        # ``input`` ops only declare parameters (reference function.py:105-115).
        if op.name == "input":
            return
        self._block.add_op(op)

    def get_value(self, name: str) -> Optional[Value]:
        for v in self._inputs:
            if v.name == name:
                return v
        return self._block.get_value(name)

    @staticmethod
    def generate_name(prefix: str = "v") -> str:
        return f"%{prefix}{next(Function._names)}"

    def __repr__(self) -> str:
        lines = [f"func @{self._name}("]
        if self._inputs:
            lines.append("  inputs: " + ", ".join(f"{v.name} : {v.type!r}" for v in self._inputs))
        else:
            lines.append("  inputs: ()")
        lines.append("  {")
        lines += [f"    {op}" for op in self._block.ops]
        lines.append("  }")
        if self._outputs:
            lines.append("  return " + ", ".join(f"{v.name} : {v.type!r}" for v in self._outputs))
        else:
            lines.append("  return (none)")
        lines.append(")")
        return "\n".join(lines)
