"""Type system of the DevProc IR.

Mirrors the reference's strict type system (src/devproc/ir/types.py:10-236):
every value is typed, shapes are tuples of positive ints, dtypes come from a
closed set.  This build adds ``bfloat16`` (absent from the reference's set at
types.py:139-142) because the bf16 pipelines store bf16 tensors.
"""

from typing import Optional, Tuple

# Element sizes in bytes; the closed dtype set of TensorType.
DTYPE_BYTES = {
    "uint8": 1, "int8": 1, "bool": 1,
    "int16": 2, "float16": 2, "bfloat16": 2,
    "int32": 4, "float32": 4,
    "int64": 8, "float64": 8,
}

FLOAT_DTYPES = frozenset(["float16", "bfloat16", "float32", "float64"])
INT_DTYPES = frozenset(["uint8", "int8", "int16", "int32", "int64", "bool"])


class Type:
    """Base class of all IR types; equality is structural per subclass."""

    def __repr__(self) -> str:
        return type(self).__name__

    def __eq__(self, other) -> bool:
        return isinstance(other, type(self)) and self._key() == other._key()

    def __hash__(self) -> int:
        return hash((type(self).__name__, self._key()))

    def _key(self):
        raise NotImplementedError


class StringType(Type):
    """Host string value (tokenizer pipelines; not executed on the GPU)."""

    def __init__(self, max_length: Optional[int] = None):
        self._max_length = max_length

    @property
    def max_length(self) -> Optional[int]:
        return self._max_length

    def _key(self):
        return (self._max_length,)

    def __repr__(self) -> str:
        return f"string[{self._max_length}]" if self._max_length else "string"


class TokenizerType(Type):
    """Host tokenizer handle (reference types.py:53-73)."""

    def __init__(self, tokenizer_name: str = "unknown"):
        self._tokenizer_name = tokenizer_name

    @property
    def tokenizer_name(self) -> str:
        return self._tokenizer_name

    def _key(self):
        return (self._tokenizer_name,)

    def __repr__(self) -> str:
        return f"tokenizer[{self._tokenizer_name}]"


class DictType(Type):
    """Host dictionary type (reference types.py:76-102)."""

    def __init__(self, key_type: Type, value_type: Type):
        self._key_type = key_type
        self._value_type = value_type

    @property
    def key_type(self) -> Type:
        return self._key_type

    @property
    def value_type(self) -> Type:
        return self._value_type

    def _key(self):
        return (self._key_type, self._value_type)

    def __repr__(self) -> str:
        return f"dict<{self._key_type}, {self._value_type}>"


class ListType(Type):
    """Host list type (reference types.py:105-124)."""

    def __init__(self, element_type: Type):
        self._element_type = element_type

    @property
    def element_type(self) -> Type:
        return self._element_type

    def _key(self):
        return (self._element_type,)

    def __repr__(self) -> str:
        return f"list<{self._element_type}>"


class TensorType(Type):
    """Tensor with static shape, dtype and device.

    Validation follows reference types.py:127-195: shape must be a tuple of
    positive ints, dtype one of VALID_DTYPES, device "cpu" or "cuda".
    """

    VALID_DTYPES = frozenset(DTYPE_BYTES)
    VALID_DEVICES = frozenset(["cpu", "cuda"])

    def __init__(self, shape: Tuple[int, ...], dtype: str, device: str = "cpu"):
        if not isinstance(shape, tuple):
            raise TypeError(f"Shape must be a tuple, got {type(shape).__name__}")
        if not all(isinstance(s, int) and not isinstance(s, bool) and s > 0 for s in shape):
            raise ValueError(f"Shape must be positive integers, got {shape}")
        if not isinstance(dtype, str):
            raise TypeError(f"dtype must be a string, got {type(dtype).__name__}")
        if dtype not in self.VALID_DTYPES:
            raise ValueError(f"Invalid dtype '{dtype}'. Valid dtypes: {sorted(self.VALID_DTYPES)}")
        if not isinstance(device, str):
            raise TypeError(f"device must be a string, got {type(device).__name__}")
        if device not in self.VALID_DEVICES:
            raise ValueError(f"Invalid device '{device}'. Valid devices: {sorted(self.VALID_DEVICES)}")
        self._shape = tuple(shape)
        self._dtype = dtype
        self._device = device

    @property
    def shape(self) -> Tuple[int, ...]:
        return self._shape

    @property
    def dtype(self) -> str:
        return self._dtype

    @property
    def device(self) -> str:
        return self._device

    @property
    def numel(self) -> int:
        n = 1
        for s in self._shape:
            n *= s
        return n

    @property
    def nbytes(self) -> int:
        return self.numel * DTYPE_BYTES[self._dtype]

    def _key(self):
        return (self._shape, self._dtype, self._device)

    def __repr__(self) -> str:
        return f"{self._dtype}[{','.join(str(s) for s in self._shape)}]"


class ScalarType(Type):
    """Scalar value type (reference types.py:198-236); no uint8, no bfloat16."""

    VALID_DTYPES = frozenset(["int8", "int16", "int32", "int64", "float16",
                              "float32", "float64", "bool"])

    def __init__(self, dtype: str):
        if not isinstance(dtype, str):
            raise TypeError(f"dtype must be a string, got {type(dtype).__name__}")
        if dtype not in self.VALID_DTYPES:
            raise ValueError(f"Invalid dtype '{dtype}'. Valid dtypes: {sorted(self.VALID_DTYPES)}")
        self._dtype = dtype

    @property
    def dtype(self) -> str:
        return self._dtype

    def _key(self):
        return (self._dtype,)

    def __repr__(self) -> str:
        return f"scalar({self._dtype})"
