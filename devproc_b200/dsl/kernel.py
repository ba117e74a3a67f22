"""``@kernel``: turn a Python function into an IR Function by running it once.

Reference behaviour (src/devproc/dsl/kernel.py:83-163): the wrapper opens a
build context, turns every torch.Tensor argument into a function input named
after its parameter (shape and dtype from the tensor), runs the body — whose
DSL calls append ops — and returns the finished ``Function``.
"""

import inspect
from typing import Callable, Dict, Optional

import torch

from ..ir.base import Value
from ..ir.function import Function
from ..ir.ops import OpBuilder
from ..ir.types import TensorType

_TORCH_DTYPES = {
    torch.uint8: "uint8", torch.int8: "int8", torch.int16: "int16", torch.int32: "int32",
    torch.int64: "int64", torch.float16: "float16", torch.bfloat16: "bfloat16",
    torch.float32: "float32", torch.float64: "float64", torch.bool: "bool",
}


def torch_dtype_name(dtype: torch.dtype) -> str:
    if dtype not in _TORCH_DTYPES:
        raise TypeError(f"unsupported torch dtype {dtype}")
    return _TORCH_DTYPES[dtype]


class KernelContext:
    """The function under construction while a ``@kernel`` body runs."""

    _current: Optional["KernelContext"] = None

    def __init__(self, func_name: str):
        self.func_name = func_name
        self.ir_function = Function(func_name)
        self.param_map: Dict[str, Value] = {}
        self._output_tensor = None

    @staticmethod
    def get_current() -> "KernelContext":
        if KernelContext._current is None:
            raise RuntimeError("Not inside a @kernel function")
        return KernelContext._current

    def set_output(self, tensor: "KernelTensor") -> None:
        self._output_tensor = tensor

    def emit(self, op) -> "KernelTensor":
        """Append ``op`` to the function and wrap its first result."""
        self.ir_function.add_op(op)
        return KernelTensor(op.outputs[0])


class KernelTensor:
    """Symbolic tensor handed to a ``@kernel`` body in place of a torch.Tensor."""

    def __init__(self, ir_value: Value, name: Optional[str] = None):
        self._ir_value = ir_value
        self._name = name or ir_value.name

    @property
    def ir_value(self) -> Value:
        return self._ir_value

    @property
    def shape(self):
        return self._ir_value.type.shape

    @property
    def dtype(self):
        return self._ir_value.type.dtype

    @property
    def device(self):
        return self._ir_value.type.device

    @property
    def name(self):
        return self._name

    def __repr__(self):
        return f"KernelTensor({self._name})"


def kernel(func: Callable) -> Callable:
    """Decorator: ``func(*tensors)`` then returns the IR Function it describes."""
    params = [p.name for p in inspect.signature(func).parameters.values()
              if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD)]

    def wrapper(*args, **kwargs):
        ctx = KernelContext(func.__name__)
        prev, KernelContext._current = KernelContext._current, ctx
        try:
            wrapped = []
            for i, pname in enumerate(params):
                if i >= len(args):
                    wrapped.append(None)
                    continue
                a = args[i]
                if isinstance(a, KernelTensor):
                    wrapped.append(a)
                elif isinstance(a, torch.Tensor):
                    ttype = TensorType(tuple(int(s) for s in a.shape), torch_dtype_name(a.dtype),
                                       "cuda" if a.is_cuda else "cpu")
                    v = OpBuilder.input(pname, ttype).outputs[0]
                    ctx.ir_function.add_input(v)
                    ctx.param_map[pname] = v
                    wrapped.append(KernelTensor(v, pname))
                elif isinstance(a, str):
                    # a host string input (the text a tokenizer step encodes); the example's value is unused
                    from .ops import string_input
                    wrapped.append(string_input(pname))
                else:
                    raise TypeError(f"Expected torch.Tensor or str, got {type(a)}")
            result = func(*wrapped, **kwargs)
            if isinstance(result, KernelTensor):
                ctx.set_output(result)
                ctx.ir_function.output = result.ir_value
            elif hasattr(result, "ir_value"):  # a host value (string, dict) returned by the kernel
                ctx.ir_function.output = result.ir_value
            elif isinstance(result, (tuple, list)) and result and all(hasattr(r, "ir_value") for r in result):
                ctx.ir_function.outputs = [r.ir_value for r in result]
            return ctx.ir_function
        finally:
            KernelContext._current = prev

    wrapper.__name__ = func.__name__
    wrapper.__doc__ = func.__doc__
    wrapper.__wrapped__ = func
    return wrapper


def parse_ir(func: Callable, *example_inputs) -> Function:
    """Build the IR of a ``@kernel`` function from example tensors."""
    return func(*example_inputs)
