"""Module-level DSL operations used inside ``@kernel`` functions.

Each call appends one IR op to the current kernel context and returns a
``KernelTensor``; nothing executes.  Names and arguments follow the reference
(src/devproc/dsl/ops.py:18-327 for tensor ops, :330-655 for the host string /
tokenizer / dict ops, :657-706 for ``load_vla_module``).  Ops marked "new"
are additions this backend needs for its pipelines.
"""

from typing import Optional, Sequence, Tuple, Union

from ..ir.ops import OpBuilder
from ..ir.types import DictType, StringType, TensorType
from ..ir.base import Value
from .kernel import KernelContext, KernelTensor
from .types import MARKER_DTYPES


def _emit(op) -> KernelTensor:
    return KernelContext.get_current().emit(op)


def _dtype(d: Union[str, type]) -> str:
    if isinstance(d, type):
        if d in MARKER_DTYPES:
            return MARKER_DTYPES[d]
        raise TypeError(f"unknown dtype marker {d.__name__}")
    if hasattr(d, "is_floating_point"):  # a torch.dtype
        from .kernel import torch_dtype_name
        return torch_dtype_name(d)
    return str(d)


# ------------------------------------------------------------------ inputs
def load_image(path: str) -> KernelTensor:
    """Placeholder image input fixed at uint8[224,224,3] (reference ops.py:18-43)."""
    ctx = KernelContext.get_current()
    v = OpBuilder.input(f"img_{path}", TensorType((224, 224, 3), "uint8", "cpu")).outputs[0]
    if v.name not in ctx.param_map:
        ctx.ir_function.add_input(v)
        ctx.param_map[v.name] = v
    return KernelTensor(v, v.name)


def input(name: str, dtype: str, shape: Tuple[int, ...], device: str = "cpu") -> KernelTensor:
    ctx = KernelContext.get_current()
    v = OpBuilder.input(name, TensorType(tuple(shape), _dtype(dtype), device)).outputs[0]
    ctx.ir_function.add_input(v)
    ctx.param_map[name] = v
    return KernelTensor(v, name)


# -------------------------------------------------------- preprocessing
def to(tensor: KernelTensor, dtype, device: Optional[str] = None) -> KernelTensor:
    return _emit(OpBuilder.to(tensor.ir_value, _dtype(dtype), device))


def normalize(tensor: KernelTensor, mean: Optional[Sequence[float]] = None,
              std: Optional[Sequence[float]] = None, channel_dim: int = -1) -> KernelTensor:
    """fp32 cast; with mean/std also ``(x - mean[c]) / std[c]`` (new arguments)."""
    return _emit(OpBuilder.normalize(tensor.ir_value, mean, std, channel_dim))


def resize(tensor: KernelTensor, size: Tuple[int, ...], layout: Optional[str] = None) -> KernelTensor:
    return _emit(OpBuilder.resize(tensor.ir_value, size, layout=layout))


def transpose(tensor: KernelTensor, dims: Tuple[int, ...]) -> KernelTensor:
    return _emit(OpBuilder.transpose(tensor.ir_value, dims))


def reshape(tensor: KernelTensor, shape: Tuple[int, ...]) -> KernelTensor:
    """new: view with a new static shape."""
    return _emit(OpBuilder.reshape(tensor.ir_value, shape))


# ------------------------------------------------------------ networks
def matmul(a: KernelTensor, b: KernelTensor) -> KernelTensor:
    return _emit(OpBuilder.matmul(a.ir_value, b.ir_value))


def linear(input: KernelTensor, weight: KernelTensor, bias: Optional[KernelTensor] = None) -> KernelTensor:
    return _emit(OpBuilder.linear(input.ir_value, weight.ir_value,
                                  bias.ir_value if bias is not None else None))


def relu(tensor: KernelTensor) -> KernelTensor:
    return _emit(OpBuilder.relu(tensor.ir_value))


def sigmoid(tensor: KernelTensor) -> KernelTensor:
    return _emit(OpBuilder.sigmoid(tensor.ir_value))


def gelu(tensor: KernelTensor, approximate: str = "none") -> KernelTensor:
    """new: GELU, exact (erf) or tanh approximation."""
    return _emit(OpBuilder.gelu(tensor.ir_value, approximate))


def tanh(tensor: KernelTensor) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.unary("tanh", tensor.ir_value))


def silu(tensor: KernelTensor) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.unary("silu", tensor.ir_value))


def exp(tensor: KernelTensor) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.unary("exp", tensor.ir_value))


def softmax(tensor: KernelTensor, dim: int = -1) -> KernelTensor:
    return _emit(OpBuilder.softmax(tensor.ir_value, dim))


def add(a: KernelTensor, b: KernelTensor) -> KernelTensor:
    return _emit(OpBuilder.add(a.ir_value, b.ir_value))


def sub(a: KernelTensor, b: KernelTensor) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.binary("sub", a.ir_value, b.ir_value))


def mul(a: KernelTensor, b: KernelTensor) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.binary("mul", a.ir_value, b.ir_value))


def div(a: KernelTensor, b: KernelTensor) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.binary("div", a.ir_value, b.ir_value))


def argmax(tensor: KernelTensor, dim: int = -1, dtype: Optional[str] = None) -> KernelTensor:
    """Row argmax; ``dtype`` ("int32"/"int64", new) gives a tensor result type."""
    return _emit(OpBuilder.argmax(tensor.ir_value, dim, _dtype(dtype) if dtype else None))


def sum(tensor: KernelTensor, dim: int = -1, keepdim: bool = False) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.reduce("sum", tensor.ir_value, dim, keepdim))


def max(tensor: KernelTensor, dim: int = -1, keepdim: bool = False) -> KernelTensor:
    """new: maximum values along ``dim``."""
    return _emit(OpBuilder.reduce("max", tensor.ir_value, dim, keepdim))


def mean(tensor: KernelTensor, dim: int = -1, keepdim: bool = False) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.reduce("mean", tensor.ir_value, dim, keepdim))


def layer_norm(tensor: KernelTensor, weight: Optional[KernelTensor] = None,
               bias: Optional[KernelTensor] = None, eps: float = 1e-5) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.layer_norm(tensor.ir_value, weight.ir_value if weight else None,
                                      bias.ir_value if bias else None, eps))


def rms_norm(tensor: KernelTensor, weight: Optional[KernelTensor] = None,
             eps: float = 1e-6) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.rms_norm(tensor.ir_value, weight.ir_value if weight else None, eps))


def embedding(ids: KernelTensor, weight: KernelTensor) -> KernelTensor:
    """new."""
    return _emit(OpBuilder.embedding(ids.ir_value, weight.ir_value))


def sdpa(q: KernelTensor, k: KernelTensor, v: KernelTensor, scale: Optional[float] = None) -> KernelTensor:
    """new: softmax(q·kᵀ·scale)·v; k / v may have fewer heads (grouped-query)."""
    return _emit(OpBuilder.sdpa(q.ir_value, k.ir_value, v.ir_value, scale))


def slice(tensor: KernelTensor, dim: int, start: int, end: int, step: int = 1) -> KernelTensor:
    """new: tensor[..., start:end:step, ...] along ``dim`` (a view)."""
    return _emit(OpBuilder.slice(tensor.ir_value, dim, start, end, step))


def cat(tensors: Sequence[KernelTensor], dim: int = 0) -> KernelTensor:
    """new: concatenation along ``dim``."""
    return _emit(OpBuilder.cat([t.ir_value for t in tensors], dim))


def rope(tensor: KernelTensor, cos: KernelTensor, sin: KernelTensor) -> KernelTensor:
    """new: rotate-half rotary embedding, tensor·cos + [-x2, x1]·sin."""
    return _emit(OpBuilder.rope(tensor.ir_value, cos.ir_value, sin.ir_value))


# ------------------------------------------------ host-side value kinds
class _HostHandle:
    def __init__(self, ir_value: Value, name: Optional[str] = None):
        self._ir_value = ir_value
        self._name = name or ir_value.name

    @property
    def ir_value(self) -> Value:
        return self._ir_value

    @property
    def name(self) -> str:
        return self._name


class KernelString(_HostHandle):
    """String handle inside a kernel body."""


class KernelTokenizer(_HostHandle):
    """Tokenizer handle inside a kernel body."""


class KernelDict(_HostHandle):
    """Dict handle inside a kernel body."""


def _append(op):
    KernelContext.get_current().ir_function.add_op(op)
    return op.outputs[0]


def load_tokenizer(tokenizer_path: str) -> KernelTokenizer:
    return KernelTokenizer(_append(OpBuilder.load_tokenizer(tokenizer_path)),
                           f"tokenizer_{tokenizer_path}")


def tokenize_encode(tokenizer: KernelTokenizer, text: KernelString) -> KernelTensor:
    return KernelTensor(_append(OpBuilder.tokenize_encode(tokenizer.ir_value, text.ir_value)))


def tokenize_decode(tokenizer: KernelTokenizer, token_ids: KernelTensor) -> KernelString:
    return KernelString(_append(OpBuilder.tokenize_decode(tokenizer.ir_value, token_ids.ir_value)))


def string_input(name: str, max_length: Optional[int] = None) -> KernelString:
    ctx = KernelContext.get_current()
    v = Value(name, StringType(max_length))
    ctx.ir_function.add_input(v)
    ctx.param_map[name] = v
    return KernelString(v, name)


def string_length(text: KernelString) -> KernelTensor:
    return KernelTensor(_append(OpBuilder.string_length(text.ir_value)))


def string_concat(a: KernelString, b: KernelString) -> KernelString:
    return KernelString(_append(OpBuilder.string_concat(a.ir_value, b.ir_value)))


def string_slice(text: KernelString, start: int, end: Optional[int] = None) -> KernelString:
    return KernelString(_append(OpBuilder.string_slice(text.ir_value, start, end)))


def string_format(template: KernelString, *args: KernelTensor) -> KernelString:
    return KernelString(_append(OpBuilder.string_format(template.ir_value,
                                                        *[a.ir_value for a in args])))


def _dict_side(kind: str):
    return StringType() if kind == "string" else TensorType((), kind, "cpu")


def dict_create(key_dtype: str, value_dtype: str) -> KernelDict:
    return KernelDict(_append(OpBuilder.dict_create(_dict_side(key_dtype), _dict_side(value_dtype))))


def dict_get(d: KernelDict, key: KernelString) -> KernelTensor:
    return KernelTensor(_append(OpBuilder.dict_get(d.ir_value, key.ir_value)))


def dict_set(d: KernelDict, key: KernelString, value: KernelTensor) -> KernelDict:
    return KernelDict(_append(OpBuilder.dict_set(d.ir_value, key.ir_value, value.ir_value)))


def dict_size(d: KernelDict) -> KernelTensor:
    return KernelTensor(_append(OpBuilder.dict_size(d.ir_value)))


def load_vla_module(model_path: str):
    """Load a LeRobot pi0.5 policy's torch module (reference ops.py:657-706).

    ``lerobot`` is an optional dependency; without it this raises ImportError,
    as the reference does.
    """
    try:
        from lerobot.policies.pi05 import PI05Policy  # type: ignore
    except ImportError as e:
        raise ImportError("LeRobot is required to load VLA models") from e
    try:
        return PI05Policy.from_pretrained(model_path).model
    except Exception as e:  # pragma: no cover - needs checkpoints
        raise RuntimeError(f"Failed to load VLA model from {model_path}: {e}") from e
