"""SSA values and operations of the DevProc IR.

Same contract as the reference (src/devproc/ir/base.py:14-137): a Value is
defined once, records the ops that use it, and an Op lists its input and
output Values.  Op attributes live in ``op.attrs``; the reference's ad-hoc
attributes (``_size``, ``_dims``, ``_dtype``, ``_device``, ``_dim``) are kept
as mirrors so code written against the reference keeps reading them.
"""

from typing import Any, Dict, List, Optional


class Value:
    """A typed SSA value; ``op`` is None for function inputs."""

    def __init__(self, name: str, type, op: Optional["Op"] = None):
        self._name = name
        self._type = type
        self._op = op
        self._uses: List["Op"] = []

    @property
    def name(self) -> str:
        return self._name

    @property
    def type(self):
        return self._type

    @property
    def op(self) -> Optional["Op"]:
        return self._op

    @property
    def uses(self) -> List["Op"]:
        return self._uses

    def add_use(self, op: "Op") -> None:
        if op not in self._uses:
            self._uses.append(op)

    def __repr__(self) -> str:
        return self._name

    def __str__(self) -> str:
        return f"{self._name} : {self._type!r}"


# Attribute names the reference printed (base.py:111-128), in its order.
_LEGACY_ATTRS = ("size", "dims", "dtype", "device", "dim")


class Op:
    """An IR operation: name, input Values, output Values, attributes."""

    def __init__(self, name: str, inputs: List[Value], outputs: List[Value],
                 attrs: Optional[Dict[str, Any]] = None):
        self._name = name
        self._inputs = list(inputs)
        self._outputs = list(outputs)
        self.attrs: Dict[str, Any] = {}
        for v in self._inputs:
            v.add_use(self)
        for v in self._outputs:
            if v._op is None:
                v._op = self
        for k, v in (attrs or {}).items():
            self.set_attr(k, v)

    def set_attr(self, key: str, value: Any) -> None:
        self.attrs[key] = value
        if key in _LEGACY_ATTRS:
            setattr(self, "_" + key, value)

    def attr(self, key: str, default: Any = None) -> Any:
        return self.attrs.get(key, default)

    @property
    def name(self) -> str:
        return self._name

    @property
    def inputs(self) -> List[Value]:
        return self._inputs

    @property
    def outputs(self) -> List[Value]:
        return self._outputs

    def _add_output(self, value: Value) -> None:
        self._outputs.append(value)

    def _get_attrs_str(self) -> str:
        parts = [f"{k}={self.attrs[k]}" for k in _LEGACY_ATTRS if k in self.attrs]
        parts += [f"{k}={v}" for k, v in self.attrs.items() if k not in _LEGACY_ATTRS]
        return f"[{', '.join(parts)}]" if parts else ""

    def __repr__(self) -> str:
        outs = ", ".join(f"{v.name} : {v.type!r}" for v in self._outputs)
        ins = ", ".join(v.name for v in self._inputs)
        return f"{outs} = {self._name}{self._get_attrs_str()}({ins})"

    __str__ = __repr__
