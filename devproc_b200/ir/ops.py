"""Op builders of the DevProc IR.

``OpBuilder`` keeps the reference's builder names and argument meanings
(src/devproc/ir/ops.py:17-618) and fixes the shape rules that the reference
got wrong for the pipelines this backend runs:

* ``normalize`` takes optional per-channel ``mean``/``std`` (the reference
  only casts, ops.py:36-57); without them it is still the plain fp32 cast.
* ``argmax`` keeps the reference's ``scalar(int64)`` result when called as
  before (ops.py:60-82); with ``dtype=`` it returns a tensor of the reduced
  shape.  Either way the backend writes one index per reduced row.
* ``matmul`` accepts batched operands; ``linear`` flattens leading dims
  (reference ops.py:131-135 kept only ``shape[0]``).
* ``add``/``sub``/``mul``/``div`` broadcast (reference ops.py:187-192 raised).
* ``resize`` handles HWC, NHWC and NCHW; an integer image resizes to float32,
  because the interpolation is defined in fp32 with no rounding back to the
  integer type (the reference kept uint8 at ops.py:235-238).

New ops needed by the pipelines: gelu, tanh, silu, exp, neg, sum, max, mean,
layer_norm, rms_norm, embedding, reshape, sdpa, slice, expand, cat, rope.
"""

import builtins
from typing import Optional, Sequence, Tuple

from .base import Op, Value
from .function import Function
from .types import (FLOAT_DTYPES, DictType, ScalarType, StringType, TensorType,
                    TokenizerType, Type)


builtins_slice = builtins.slice


def _tensor(v: Value, opname: str) -> TensorType:
    if not isinstance(v.type, TensorType):
        raise TypeError(f"{opname} requires TensorType, got {type(v.type)}")
    return v.type


def _new(t: Type) -> Value:
    return Value(Function.generate_name(), t)


def _norm_dim(dim: int, rank: int) -> int:
    d = dim + rank if dim < 0 else dim
    if not 0 <= d < max(rank, 1):
        raise ValueError(f"dim {dim} out of range for rank {rank}")
    return d


def broadcast_shapes(a: Tuple[int, ...], b: Tuple[int, ...]) -> Tuple[int, ...]:
    """Numpy broadcasting of two static shapes."""
    out = []
    for i in range(max(len(a), len(b))):
        x = a[len(a) - 1 - i] if i < len(a) else 1
        y = b[len(b) - 1 - i] if i < len(b) else 1
        if x != y and x != 1 and y != 1:
            raise ValueError(f"shapes {a} and {b} do not broadcast")
        out.append(max(x, y))
    return tuple(reversed(out))


_PROMOTE_ORDER = ["bool", "uint8", "int8", "int16", "int32", "int64",
                  "float16", "bfloat16", "float32", "float64"]


def promote(a: str, b: str) -> str:
    """Result dtype of a binary elementwise op (fp16+bf16 → fp32, as torch)."""
    if {a, b} == {"float16", "bfloat16"}:
        return "float32"
    return a if _PROMOTE_ORDER.index(a) >= _PROMOTE_ORDER.index(b) else b


class OpBuilder:
    """Static constructors for every IR op (no execution happens here)."""

    # ------------------------------------------------------------- inputs
    @staticmethod
    def input(name: str, tensor_type: Type) -> Op:
        return Op("input", [], [Value(name, tensor_type)])

    @staticmethod
    def return_op(value: Value) -> Op:
        return Op("return", [value], [])

    # ------------------------------------------------------ preprocessing
    @staticmethod
    def normalize(x: Value, mean: Optional[Sequence[float]] = None,
                  std: Optional[Sequence[float]] = None, channel_dim: int = -1) -> Op:
        """fp32 cast, then ``(x - mean[c]) / std[c]`` when mean/std are given.

        ``c`` indexes ``channel_dim`` (the last dim for HWC/NHWC images).
        """
        t = _tensor(x, "normalize")
        attrs = {}
        if mean is not None or std is not None:
            rank = len(t.shape)
            cd = _norm_dim(channel_dim, rank)
            nch = t.shape[cd]
            mean = [float(m) for m in (mean if mean is not None else [0.0] * nch)]
            std = [float(s) for s in (std if std is not None else [1.0] * nch)]
            if len(mean) != nch or len(std) != nch:
                raise ValueError(f"normalize: mean/std need {nch} channels")
            if any(s == 0.0 for s in std):
                raise ValueError("normalize: std must be non-zero")
            attrs = {"mean": tuple(mean), "std": tuple(std), "channel_dim": cd}
        return Op("normalize", [x], [_new(TensorType(t.shape, "float32", t.device))], attrs)

    @staticmethod
    def resize(x: Value, size: Tuple[int, ...], mode: str = "bilinear",
               layout: Optional[str] = None) -> Op:
        """Bilinear resize (align_corners=False) of the spatial dims.

        ``layout`` defaults to HWC for rank 3 and NHWC for rank 4; "NCHW" and
        "CHW" are also accepted (FX ``interpolate`` produces NCHW).
        """
        t = _tensor(x, "resize")
        size = tuple(int(s) for s in size)
        rank = len(t.shape)
        if mode != "bilinear":
            raise ValueError(f"resize: only bilinear is supported, got {mode}")
        if layout is None:
            layout = {3: "HWC", 4: "NHWC", 2: "HW"}.get(rank)
        if layout not in ("HWC", "NHWC", "NCHW", "CHW", "HW") or len(layout) != rank:
            raise ValueError(f"resize: unsupported layout {layout} for rank {rank}")
        if len(size) != 2:
            raise ValueError(f"resize: size must be (H, W), got {size}")
        shape = list(t.shape)
        shape[layout.index("H")] = size[0]
        shape[layout.index("W")] = size[1]
        dtype = t.dtype if t.dtype in FLOAT_DTYPES else "float32"
        return Op("resize", [x], [_new(TensorType(tuple(shape), dtype, t.device))],
                  {"size": size, "mode": mode, "layout": layout})

    @staticmethod
    def transpose(x: Value, dims: Tuple[int, ...]) -> Op:
        """Permute dims; a 2-element ``dims`` on a higher-rank tensor swaps those two."""
        t = _tensor(x, "transpose")
        rank = len(t.shape)
        dims = tuple(int(d) for d in dims)
        if len(dims) == 2 and rank != 2:
            a, b = (_norm_dim(d, rank) for d in dims)
            perm = list(range(rank))
            perm[a], perm[b] = perm[b], perm[a]
            dims = tuple(perm)
        dims = tuple(_norm_dim(d, rank) for d in dims)
        if sorted(dims) != list(range(rank)):
            raise ValueError(f"transpose: {dims} is not a permutation of rank {rank}")
        shape = tuple(t.shape[d] for d in dims)
        return Op("transpose", [x], [_new(TensorType(shape, t.dtype, t.device))], {"dims": dims})

    @staticmethod
    def slice(x: Value, dim: int, start: int, end: int, step: int = 1) -> Op:
        """x[..., start:end:step, ...] along ``dim`` (Python slice bounds, clamped)."""
        t = _tensor(x, "slice")
        d = _norm_dim(dim, len(t.shape))
        if step < 1:
            raise ValueError("slice: step must be positive")
        start, end, step = builtins_slice(start, end, step).indices(t.shape[d])
        n = len(range(start, end, step))
        shape = tuple(n if i == d else s for i, s in enumerate(t.shape))
        return Op("slice", [x], [_new(TensorType(shape, t.dtype, t.device))],
                  {"dim": d, "start": start, "end": end, "step": step})

    @staticmethod
    def expand(x: Value, shape: Tuple[int, ...]) -> Op:
        """Broadcast ``x`` to ``shape`` (torch ``expand``; -1 keeps a dim)."""
        t = _tensor(x, "expand")
        shape = tuple(int(s) for s in shape)
        lead = len(shape) - len(t.shape)
        if lead < 0:
            raise ValueError("expand: fewer dims than the input")
        full = []
        for i, s in enumerate(shape):
            src = t.shape[i - lead] if i >= lead else 1
            s = src if s == -1 else s
            if src != s and src != 1:
                raise ValueError(f"expand: {t.shape} cannot expand to {shape}")
            full.append(s)
        return Op("expand", [x], [_new(TensorType(tuple(full), t.dtype, t.device))], {"shape": tuple(full)})

    @staticmethod
    def cat(xs: Sequence[Value], dim: int = 0) -> Op:
        """Concatenate along ``dim``; all inputs share the other dims and the dtype."""
        ts = [_tensor(v, "cat") for v in xs]
        if not ts:
            raise ValueError("cat: no inputs")
        d = _norm_dim(dim, len(ts[0].shape))
        for t in ts[1:]:
            if len(t.shape) != len(ts[0].shape) or t.dtype != ts[0].dtype or any(
                    a != b for i, (a, b) in enumerate(zip(t.shape, ts[0].shape)) if i != d):
                raise ValueError("cat: inputs differ outside the cat dim")
        shape = tuple(sum(t.shape[d] for t in ts) if i == d else s for i, s in enumerate(ts[0].shape))
        return Op("cat", list(xs), [_new(TensorType(shape, ts[0].dtype, ts[0].device))], {"dim": d})

    @staticmethod
    def rope(x: Value, cos: Value, sin: Value) -> Op:
        """Rotary position embedding, rotate-half form: with x = [x1, x2] split
        in halves along the last dim, out = x·cos + [-x2, x1]·sin.  ``cos`` and
        ``sin`` broadcast to x and hold either the full last dim D or its half."""
        t = _tensor(x, "rope")
        tc, ts = _tensor(cos, "rope"), _tensor(sin, "rope")
        D = t.shape[-1]
        if D % 2:
            raise ValueError("rope: the last dim must be even")
        for tt in (tc, ts):
            if tt.shape[-1] not in (D, D // 2):
                raise ValueError(f"rope: cos/sin last dim {tt.shape[-1]} is neither {D} nor {D // 2}")
            broadcast_shapes(t.shape[:-1], tt.shape[:-1])
        return Op("rope", [x, cos, sin], [_new(TensorType(t.shape, t.dtype, t.device))])

    @staticmethod
    def to(x: Value, dtype: str, device: Optional[str] = None) -> Op:
        t = _tensor(x, "to")
        dev = device or t.device
        return Op("to", [x], [_new(TensorType(t.shape, dtype, dev))],
                  {"dtype": dtype, "device": dev})

    @staticmethod
    def reshape(x: Value, shape: Tuple[int, ...]) -> Op:
        t = _tensor(x, "reshape")
        shape = list(int(s) for s in shape)
        if shape.count(-1) > 1:
            raise ValueError("reshape: at most one -1")
        if -1 in shape:
            known = 1
            for s in shape:
                if s != -1:
                    known *= s
            shape[shape.index(-1)] = t.numel // known
        out = TensorType(tuple(shape), t.dtype, t.device)
        if out.numel != t.numel:
            raise ValueError(f"reshape: {t.shape} -> {tuple(shape)} changes numel")
        return Op("reshape", [x], [_new(out)], {"shape": tuple(shape)})

    # ------------------------------------------------------- contractions
    @staticmethod
    def matmul(a: Value, b: Value, out_dtype: str = "float32") -> Op:
        """C = A @ B; 2-D or batched (leading dims broadcast); fp32 result by default."""
        ta, tb = _tensor(a, "matmul"), _tensor(b, "matmul")
        if len(ta.shape) < 2 or len(tb.shape) < 2:
            raise ValueError("matmul requires tensors of rank >= 2")
        if ta.shape[-1] != tb.shape[-2]:
            raise ValueError(f"matmul dimension mismatch: {ta.shape[-1]} != {tb.shape[-2]}")
        batch = broadcast_shapes(ta.shape[:-2], tb.shape[:-2])
        shape = batch + (ta.shape[-2], tb.shape[-1])
        return Op("matmul", [a, b], [_new(TensorType(shape, out_dtype, ta.device))])

    @staticmethod
    def linear(x: Value, weight: Value, bias: Optional[Value] = None,
               out_dtype: Optional[str] = None) -> Op:
        """Y = X·Wᵀ + b over the last dim of X; W is [out_features, in_features]."""
        tx, tw = _tensor(x, "linear"), _tensor(weight, "linear")
        if len(tw.shape) != 2:
            raise ValueError("linear weight must be 2-D [out, in]")
        if tx.shape[-1] != tw.shape[1]:
            raise ValueError(f"linear: in_features {tx.shape[-1]} != weight {tw.shape[1]}")
        if bias is not None and _tensor(bias, "linear").shape != (tw.shape[0],):
            raise ValueError("linear: bias must be [out_features]")
        if out_dtype is None:
            out_dtype = tx.dtype if tx.dtype in ("bfloat16", "float16") else "float32"
        shape = tuple(tx.shape[:-1]) + (tw.shape[0],)
        ins = [x, weight] + ([bias] if bias is not None else [])
        return Op("linear", ins, [_new(TensorType(shape, out_dtype, tx.device))])

    @staticmethod
    def sdpa(q: Value, k: Value, v: Value, scale: Optional[float] = None,
             is_causal: bool = False) -> Op:
        """softmax(Q·Kᵀ·scale)·V over [..., L, D]; K/V heads may be fewer (GQA)."""
        tq, tk, tv = (_tensor(t, "sdpa") for t in (q, k, v))
        if tq.shape[-1] != tk.shape[-1] or tk.shape[-2] != tv.shape[-2]:
            raise ValueError("sdpa: shape mismatch")
        if scale is None:
            scale = tq.shape[-1] ** -0.5
        shape = tuple(tq.shape[:-1]) + (tv.shape[-1],)
        return Op("sdpa", [q, k, v], [_new(TensorType(shape, tq.dtype, tq.device))],
                  {"scale": float(scale), "is_causal": bool(is_causal)})

    # -------------------------------------------------------- elementwise
    @staticmethod
    def relu(x: Value) -> Op:
        t = _tensor(x, "relu")
        return Op("relu", [x], [_new(TensorType(t.shape, t.dtype, t.device))])

    @staticmethod
    def sigmoid(x: Value) -> Op:
        # The reference makes sigmoid's result float32 (ops.py:296-300).
        t = _tensor(x, "sigmoid")
        return Op("sigmoid", [x], [_new(TensorType(t.shape, "float32", t.device))])

    @staticmethod
    def unary(name: str, x: Value, **attrs) -> Op:
        """Same-shape, same-dtype unary ops: gelu, tanh, silu, exp, neg, abs."""
        t = _tensor(x, name)
        dtype = t.dtype if t.dtype in FLOAT_DTYPES else "float32"
        return Op(name, [x], [_new(TensorType(t.shape, dtype, t.device))], attrs)

    @staticmethod
    def gelu(x: Value, approximate: str = "none") -> Op:
        if approximate not in ("none", "tanh"):
            raise ValueError(f"gelu: approximate must be 'none' or 'tanh', got {approximate}")
        return OpBuilder.unary("gelu", x, approximate=approximate)

    @staticmethod
    def binary(name: str, a: Value, b: Value) -> Op:
        ta, tb = _tensor(a, name), _tensor(b, name)
        shape = broadcast_shapes(ta.shape, tb.shape)
        return Op(name, [a, b], [_new(TensorType(shape, promote(ta.dtype, tb.dtype), ta.device))])

    @staticmethod
    def add(a: Value, b: Value) -> Op:
        return OpBuilder.binary("add", a, b)

    @staticmethod
    def scalar_op(name: str, x: Value, scalar: float, reverse: bool = False) -> Op:
        """x (op) c, or c (op) x when ``reverse``; c is a Python float constant."""
        t = _tensor(x, name)
        dtype = t.dtype if t.dtype in FLOAT_DTYPES else "float32"
        return Op(name + "_scalar", [x], [_new(TensorType(t.shape, dtype, t.device))],
                  {"scalar": float(scalar), "reverse": bool(reverse)})

    # --------------------------------------------------------- reductions
    @staticmethod
    def softmax(x: Value, dim: int = -1) -> Op:
        t = _tensor(x, "softmax")
        return Op("softmax", [x], [_new(TensorType(t.shape, "float32", t.device))],
                  {"dim": _norm_dim(dim, len(t.shape)) - len(t.shape)})

    @staticmethod
    def argmax(x: Value, dim: int = -1, dtype: Optional[str] = None, keepdim: bool = False) -> Op:
        """Index of the first maximum along ``dim`` (NaN counts as maximum).

        ``dtype=None`` keeps the reference's scalar(int64) result type
        (ops.py:60-82); the backend still writes one int64 per reduced row.
        """
        t = _tensor(x, "argmax")
        d = _norm_dim(dim, len(t.shape))
        if dtype is None:
            out = ScalarType("int64")
        else:
            if dtype not in ("int32", "int64"):
                raise ValueError("argmax dtype must be int32 or int64")
            shape = _reduced(t.shape, d, keepdim)
            out = TensorType(shape, dtype, t.device)
        return Op("argmax", [x], [_new(out)], {"dim": d - len(t.shape), "keepdim": keepdim})

    @staticmethod
    def reduce(name: str, x: Value, dim: int = -1, keepdim: bool = False) -> Op:
        """sum / max / mean along one dim, fp32 result for fp32 input."""
        if name not in ("sum", "max", "mean", "min"):
            raise ValueError(f"unknown reduction {name}")
        t = _tensor(x, name)
        d = _norm_dim(dim, len(t.shape))
        dtype = t.dtype if t.dtype in FLOAT_DTYPES else "float32"
        shape = _reduced(t.shape, d, keepdim)
        return Op(name, [x], [_new(TensorType(shape, dtype, t.device))],
                  {"dim": d - len(t.shape), "keepdim": keepdim})

    @staticmethod
    def layer_norm(x: Value, weight: Optional[Value] = None, bias: Optional[Value] = None,
                   eps: float = 1e-5) -> Op:
        t = _tensor(x, "layer_norm")
        ins = [x] + [v for v in (weight, bias) if v is not None]
        return Op("layer_norm", ins, [_new(TensorType(t.shape, t.dtype, t.device))],
                  {"eps": float(eps), "has_weight": weight is not None,
                   "has_bias": bias is not None})

    @staticmethod
    def rms_norm(x: Value, weight: Optional[Value] = None, eps: float = 1e-6,
                 weight_offset: float = 0.0) -> Op:
        """x / sqrt(mean(x²) + eps) · (weight + weight_offset)."""
        t = _tensor(x, "rms_norm")
        ins = [x] + ([weight] if weight is not None else [])
        return Op("rms_norm", ins, [_new(TensorType(t.shape, t.dtype, t.device))],
                  {"eps": float(eps), "has_weight": weight is not None,
                   "weight_offset": float(weight_offset)})

    # -------------------------------------------------------------- misc
    @staticmethod
    def embedding(ids: Value, weight: Value) -> Op:
        ti, tw = _tensor(ids, "embedding"), _tensor(weight, "embedding")
        if ti.dtype not in ("int32", "int64"):
            raise TypeError("embedding ids must be int32 or int64")
        if len(tw.shape) != 2:
            raise ValueError("embedding weight must be 2-D")
        return Op("embedding", [ids, weight],
                  [_new(TensorType(ti.shape + (tw.shape[1],), tw.dtype, tw.device))])

    # ------------------------------------------- host ops (not GPU work)
    @staticmethod
    def load_tokenizer(tokenizer_path: str) -> Op:
        return Op("load_tokenizer", [], [_new(TokenizerType(tokenizer_path))],
                  {"tokenizer_path": tokenizer_path})

    @staticmethod
    def tokenize_encode(tokenizer: Value, text: Value) -> Op:
        if not isinstance(tokenizer.type, TokenizerType):
            raise TypeError(f"tokenize_encode requires TokenizerType, got {type(tokenizer.type)}")
        if not isinstance(text.type, StringType):
            raise TypeError(f"tokenize_encode requires StringType input, got {type(text.type)}")
        return Op("tokenize_encode", [tokenizer, text],
                  [_new(TensorType((2048,), "int32", "cpu"))], {"max_length": 2048})

    @staticmethod
    def tokenize_decode(tokenizer: Value, token_ids: Value) -> Op:
        if not isinstance(tokenizer.type, TokenizerType):
            raise TypeError(f"tokenize_decode requires TokenizerType, got {type(tokenizer.type)}")
        if not isinstance(token_ids.type, TensorType):
            raise TypeError(f"tokenize_decode requires TensorType input, got {type(token_ids.type)}")
        return Op("tokenize_decode", [tokenizer, token_ids], [_new(StringType())])

    @staticmethod
    def string_length(text: Value) -> Op:
        if not isinstance(text.type, StringType):
            raise TypeError(f"string_length requires StringType, got {type(text.type)}")
        return Op("string_length", [text], [_new(ScalarType("int32"))])

    @staticmethod
    def string_concat(a: Value, b: Value) -> Op:
        for v in (a, b):
            if not isinstance(v.type, StringType):
                raise TypeError(f"string_concat requires StringType, got {type(v.type)}")
        la, lb = a.type.max_length, b.type.max_length
        return Op("string_concat", [a, b], [_new(StringType(la + lb if la and lb else None))])

    @staticmethod
    def string_slice(text: Value, start: int, end: Optional[int] = None) -> Op:
        if not isinstance(text.type, StringType):
            raise TypeError(f"string_slice requires StringType, got {type(text.type)}")
        ml = text.type.max_length
        n = (end - start) if (ml and end) else ((ml - start) if ml else None)
        return Op("string_slice", [text], [_new(StringType(n))], {"start": start, "end": end})

    @staticmethod
    def string_format(template: Value, *args: Value) -> Op:
        if not isinstance(template.type, StringType):
            raise TypeError(f"string_format requires StringType template, got {type(template.type)}")
        return Op("string_format", [template, *args], [_new(StringType(template.type.max_length))])

    @staticmethod
    def dict_create(key_type: Type, value_type: Type) -> Op:
        return Op("dict_create", [], [_new(DictType(key_type, value_type))])

    @staticmethod
    def dict_get(d: Value, key: Value) -> Op:
        if not isinstance(d.type, DictType):
            raise TypeError(f"dict_get requires DictType, got {type(d.type)}")
        return Op("dict_get", [d, key], [_new(d.type.value_type)])

    @staticmethod
    def dict_set(d: Value, key: Value, value: Value) -> Op:
        if not isinstance(d.type, DictType):
            raise TypeError(f"dict_set requires DictType, got {type(d.type)}")
        return Op("dict_set", [d, key, value], [_new(d.type)])

    @staticmethod
    def dict_size(d: Value) -> Op:
        if not isinstance(d.type, DictType):
            raise TypeError(f"dict_size requires DictType, got {type(d.type)}")
        return Op("dict_size", [d], [_new(ScalarType("int32"))])


def _reduced(shape: Tuple[int, ...], d: int, keepdim: bool) -> Tuple[int, ...]:
    if keepdim:
        return tuple(1 if i == d else s for i, s in enumerate(shape))
    out = tuple(s for i, s in enumerate(shape) if i != d)
    return out if out else (1,)


def reduced_rows(x_type: TensorType, dim: int) -> Tuple[int, int, int]:
    """(outer, reduce_len, inner) for a reduction of ``x_type`` along ``dim``."""
    d = _norm_dim(dim, len(x_type.shape))
    outer = 1
    for s in x_type.shape[:d]:
        outer *= s
    inner = 1
    for s in x_type.shape[d + 1:]:
        inner *= s
    return outer, x_type.shape[d], inner
