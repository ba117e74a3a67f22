"""Annotation-only type markers of the ``@kernel`` DSL.

Same names as the reference (src/devproc/dsl/types.py:1-82); they carry no
behaviour.  ``to(x, Float32)`` maps a marker to its dtype string through
``MARKER_DTYPES``.  ``BFloat16`` is new in this build.
"""


class String:
    """String parameter marker."""


class Tensor:
    """Tensor parameter marker."""


class Float32:
    """float32 marker."""


class Float16:
    """float16 marker."""


class BFloat16:
    """bfloat16 marker."""


class Int32:
    """int32 marker."""


class Int64:
    """int64 marker."""


class UInt8:
    """uint8 marker."""


class Bool:
    """bool marker."""


class Tokenizer:
    """Tokenizer marker (host-side pipelines)."""


class TorchModel:
    """torch.nn.Module marker."""


class KVCache:
    """KV-cache marker."""


class IRFunction:
    """Marker for a pre-built IR Function passed into a kernel."""


MARKER_DTYPES = {
    Float32: "float32", Float16: "float16", BFloat16: "bfloat16", Int32: "int32",
    Int64: "int64", UInt8: "uint8", Bool: "bool",
}
