"""torch.fx GraphModule → DevProc IR Function.

Reference: src/devproc/ir/fx_converter.py:22-448.  Same entry point
(``FXToIRConverter().convert(gm, example_inputs)``) and the same node kinds
(placeholder, get_attr, call_function, call_method, call_module, output), with
the reference's gaps fixed:

* shapes and dtypes come from each node's ``example_value`` (Dynamo's fake
  tensor), or from the example inputs in placeholder order — the reference
  indexed ``example_inputs`` by the node's position in the whole graph
  (fx_converter.py:115-124), which gave wrong shapes as soon as parameters
  were lifted to placeholders;
* placeholders whose example input is an ``nn.Parameter`` or buffer become
  *constants* of the function (``fn.constants``): the compiled program
  uploads them once instead of taking them as per-call inputs;
* call arguments that are Python values (dims, eps, dtypes, sizes) are read;
* embedding, gelu, layer_norm, rms_norm, softmax, mean/sum/max, interpolate,
  permute/transpose/view/reshape/flatten, scalar arithmetic and
  conv2d-as-patchify are lowered; anything else raises ``ValueError`` naming
  the op (the reference silently built a same-shape placeholder op,
  fx_converter.py:443-448).
"""

import operator
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.fx

from .base import Value
from .function import Function
from .ops import OpBuilder
from .types import TensorType
from .fx_op_map import get_fx_op_map

_DT = {torch.uint8: "uint8", torch.int8: "int8", torch.int16: "int16", torch.int32: "int32",
       torch.int64: "int64", torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32",
       torch.float64: "float64", torch.bool: "bool"}


def _ttype(t: torch.Tensor) -> TensorType:
    if t.dtype not in _DT:
        raise ValueError(f"unsupported dtype {t.dtype}")
    return TensorType(tuple(int(s) for s in t.shape), _DT[t.dtype], "cuda" if t.is_cuda else "cpu")


def _meta_val(node):
    """The node's example result: Dynamo's ``example_value``, or ``val`` in a torch.export graph."""
    ev = node.meta.get("example_value")
    return node.meta.get("val") if ev is None else ev


def _target_name(target) -> str:
    if isinstance(target, str):
        return target
    if isinstance(target, torch._ops.OpOverload):  # aten.add.Tensor → "add"
        return target.overloadpacket.__name__
    name = getattr(target, "__name__", None) or str(target)
    if name.endswith(".default"):
        name = name[:-8]
    return name


@dataclass
class FXToIRConverter:
    op_map: Dict[str, str] = field(default_factory=get_fx_op_map)
    value_map: Dict[Any, Value] = field(default_factory=dict)
    tuple_map: Dict[Any, List[Value]] = field(default_factory=dict)  # split / chunk results
    gm: Optional[torch.fx.GraphModule] = field(default=None, init=False)
    example_inputs: Tuple[Any, ...] = field(default_factory=tuple, init=False)

    def convert(self, gm: torch.fx.GraphModule, example_inputs: Tuple[Any, ...]) -> Function:
        self.gm = gm
        self.example_inputs = tuple(example_inputs)
        self.value_map = {}
        self.tuple_map = {}
        self.fn = Function(type(gm).__name__ if gm is not None else "fx_graph")
        self.fn.constants = {}
        self._ph_index = 0
        for node in gm.graph.nodes:
            handler = getattr(self, "_on_" + node.op, None)
            if handler is None:
                raise ValueError(f"Unsupported FX node op: {node.op}")
            handler(node)
        return self.fn

    # ------------------------------------------------------------ helpers
    def _v(self, a) -> Value:
        if isinstance(a, torch.fx.Node):
            if a not in self.value_map:
                raise ValueError(f"FX node {a.name} has no IR value")
            return self.value_map[a]
        raise ValueError(f"expected a tensor argument, got {a!r}")

    def _emit(self, node: torch.fx.Node, op) -> Value:
        self.fn.block.add_op(op)
        out = op.outputs[0]
        ev = _meta_val(node) if node is not None else None
        if isinstance(ev, torch.Tensor) and isinstance(out.type, TensorType):
            if tuple(ev.shape) != out.type.shape:
                raise ValueError(f"shape rule mismatch at {node.name} ({op.name}): IR {out.type.shape} vs "
                                 f"torch {tuple(ev.shape)}")
        if node is not None:
            self.value_map[node] = out
        return out

    def _add_input(self, node, name: str, example, is_const: bool) -> None:
        ttype = _ttype(example)
        v = OpBuilder.input(name, ttype).outputs[0]
        self.fn.add_input(v)
        if is_const:
            self.fn.constants[name] = example.detach()
        self.value_map[node] = v

    @staticmethod
    def _arg(node, i, key, default=None):
        if len(node.args) > i:
            return node.args[i]
        return node.kwargs.get(key, default)

    def _ex_shape(self, node) -> Tuple[int, ...]:
        ev = _meta_val(node)
        if isinstance(ev, torch.Tensor):
            return tuple(int(s) for s in ev.shape)
        raise ValueError(f"{node.name}: no example_value to take the result shape from")

    # ------------------------------------------------------------- nodes
    def _on_placeholder(self, node) -> None:
        idx = self._ph_index
        self._ph_index += 1
        example = self.example_inputs[idx] if idx < len(self.example_inputs) else None
        if not isinstance(example, torch.Tensor):
            ev = _meta_val(node)
            if not isinstance(ev, torch.Tensor):
                raise ValueError(f"placeholder {node.name}: no tensor example")
            example = ev
        is_const = isinstance(example, torch.nn.Parameter) or "_buffers_" in node.name
        self._add_input(node, node.name, example, is_const)

    def _on_get_attr(self, node) -> None:
        obj = self.gm
        for part in node.target.split("."):
            obj = getattr(obj, part)
        if not isinstance(obj, torch.Tensor):
            raise ValueError(f"Unsupported get_attr target: {node.target}, type: {type(obj)}")
        self._add_input(node, node.name, obj, True)

    def _on_call_module(self, node) -> None:
        mod = self.gm.get_submodule(node.target)
        x = self._v(node.args[0])
        prefix = node.target.replace(".", "_")

        def const(t, suffix):
            name = f"{prefix}_{suffix}"
            v = OpBuilder.input(name, _ttype(t)).outputs[0]
            self.fn.add_input(v)
            self.fn.constants[name] = t.detach()
            return v

        if isinstance(mod, torch.nn.Linear):
            b = const(mod.bias, "bias") if mod.bias is not None else None
            self._emit(node, OpBuilder.linear(x, const(mod.weight, "weight"), b))
        elif isinstance(mod, torch.nn.ReLU):
            self._emit(node, OpBuilder.relu(x))
        elif isinstance(mod, torch.nn.GELU):
            self._emit(node, OpBuilder.gelu(x, mod.approximate))
        elif isinstance(mod, torch.nn.Sigmoid):
            self._emit(node, OpBuilder.sigmoid(x))
        elif isinstance(mod, torch.nn.LayerNorm):
            w = const(mod.weight, "weight") if mod.weight is not None else None
            b = const(mod.bias, "bias") if mod.bias is not None else None
            self._emit(node, OpBuilder.layer_norm(x, w, b, mod.eps))
        elif isinstance(mod, torch.nn.Embedding):
            self._emit(node, OpBuilder.embedding(x, const(mod.weight, "weight")))
        elif isinstance(mod, torch.nn.Softmax):
            self._emit(node, OpBuilder.softmax(x, mod.dim if mod.dim is not None else -1))
        else:
            raise ValueError(f"Unsupported module type: {type(mod)}")

    def _on_call_method(self, node) -> None:
        self._dispatch(node, node.target, node.args, node.kwargs)

    def _on_call_function(self, node) -> None:
        t = node.target
        if t is operator.getitem:
            return self._getitem(node)
        self._dispatch(node, _target_name(t), node.args, node.kwargs)

    def _getitem(self, node) -> None:
        """``tuple[i]`` of a split/chunk result, or tensor indexing with ints,
        slices, ``None`` and ``...`` (basic indexing: views, no gathers)."""
        src, idx = node.args
        if src in self.tuple_map:
            self.value_map[node] = self.tuple_map[src][idx]
            return
        x = self._v(src)
        items = list(idx) if isinstance(idx, tuple) else [idx]
        rank = len(x.type.shape)
        n_real = sum(1 for it in items if it is not None and it is not Ellipsis)
        if n_real > rank:
            raise ValueError(f"getitem {node.name}: too many indices")
        if Ellipsis in items:
            e = items.index(Ellipsis)
            items = items[:e] + [slice(None)] * (rank - n_real) + items[e + 1:]
        items += [slice(None)] * (rank - sum(1 for it in items if it is not None))
        cur, d = x, 0
        squeeze, unsqueeze = [], []
        out_pos = 0
        for it in items:
            if it is None:
                unsqueeze.append(out_pos)
                out_pos += 1
                continue
            if isinstance(it, int):
                size = cur.type.shape[d]
                i = it + size if it < 0 else it
                if not 0 <= i < size:
                    raise ValueError(f"getitem {node.name}: index {it} out of range")
                op = OpBuilder.slice(cur, d, i, i + 1)
                self.fn.block.add_op(op)
                cur = op.outputs[0]
                squeeze.append(d)
            elif isinstance(it, slice):
                if not (it.start is None and it.stop is None and it.step in (None, 1)):
                    if any(isinstance(b, torch.fx.Node) for b in (it.start, it.stop, it.step)):
                        raise ValueError(f"getitem {node.name}: data-dependent slice bounds")
                    op = OpBuilder.slice(cur, d, 0 if it.start is None else it.start,
                                         cur.type.shape[d] if it.stop is None else it.stop, it.step or 1)
                    self.fn.block.add_op(op)
                    cur = op.outputs[0]
                out_pos += 1
            else:
                raise ValueError(f"getitem {node.name}: unsupported index {it!r} (tensor indexing)")
            d += 1
        shape = self._ex_shape(node)
        if tuple(cur.type.shape) != shape:
            cur = self._reshape_value(cur, shape)
        self.value_map[node] = cur

    def _on_output(self, node) -> None:
        res = node.args[0]
        items = list(res) if isinstance(res, (tuple, list)) else [res]
        outs = []
        for it in items:
            if not isinstance(it, torch.fx.Node):
                raise ValueError(f"non-tensor graph output {it!r}")
            outs.append(self._v(it))
        self.fn.outputs = outs

    # ----------------------------------------------------------- dispatch
    def _dispatch(self, node, name: str, args, kwargs) -> None:
        ir = self.op_map.get(name)
        if ir is None:
            raise ValueError(f"Unsupported FX function: {name}")
        getattr(self, "_op_" + ir)(node, args, kwargs)

    def _op_passthrough(self, node, args, kwargs):
        self.value_map[node] = self._v(args[0])

    def _op_linear(self, node, args, kwargs):
        b = self._arg(node, 2, "bias")
        self._emit(node, OpBuilder.linear(self._v(args[0]), self._v(self._arg(node, 1, "weight")),
                                          self._v(b) if b is not None else None))

    def _op_matmul(self, node, args, kwargs):
        a, b = self._v(args[0]), self._v(args[1])
        ev = _meta_val(node)
        out = _DT[ev.dtype] if isinstance(ev, torch.Tensor) else "float32"
        self._emit(node, OpBuilder.matmul(a, b, out_dtype=out))

    def _op_embedding(self, node, args, kwargs):
        self._emit(node, OpBuilder.embedding(self._v(args[0]), self._v(args[1])))

    def _op_unary(self, node, args, kwargs, name):
        x = self._v(args[0])
        if name == "relu":
            self._emit(node, OpBuilder.relu(x))
        elif name == "sigmoid":
            self._emit(node, OpBuilder.sigmoid(x))
        else:
            self._emit(node, OpBuilder.unary(name, x))

    def _op_relu(self, node, args, kwargs):
        self._op_unary(node, args, kwargs, "relu")

    def _op_sigmoid(self, node, args, kwargs):
        self._op_unary(node, args, kwargs, "sigmoid")

    def _op_tanh(self, node, args, kwargs):
        self._op_unary(node, args, kwargs, "tanh")

    def _op_silu(self, node, args, kwargs):
        self._op_unary(node, args, kwargs, "silu")

    def _op_exp(self, node, args, kwargs):
        self._op_unary(node, args, kwargs, "exp")

    def _op_neg(self, node, args, kwargs):
        self._op_unary(node, args, kwargs, "neg")

    def _op_gelu(self, node, args, kwargs):
        approx = kwargs.get("approximate", args[1] if len(args) > 1 else "none")
        self._emit(node, OpBuilder.gelu(self._v(args[0]), approx))

    def _binary(self, node, args, name):
        a, b = args[0], args[1]
        if isinstance(a, torch.fx.Node) and isinstance(b, torch.fx.Node):
            self._emit(node, OpBuilder.binary(name, self._v(a), self._v(b)))
        elif isinstance(a, torch.fx.Node):
            self._emit(node, OpBuilder.scalar_op(name, self._v(a), float(b)))
        elif isinstance(b, torch.fx.Node):
            self._emit(node, OpBuilder.scalar_op(name, self._v(b), float(a), reverse=True))
        else:
            raise ValueError(f"{name} of two constants")

    def _op_add(self, node, args, kwargs):
        if kwargs.get("alpha", 1) != 1:
            raise ValueError("add with alpha is not supported")
        self._binary(node, args, "add")

    def _op_sub(self, node, args, kwargs):
        self._binary(node, args, "sub")

    def _op_mul(self, node, args, kwargs):
        self._binary(node, args, "mul")

    def _op_div(self, node, args, kwargs):
        if kwargs.get("rounding_mode") is not None:
            raise ValueError("div with rounding_mode is not supported")
        self._binary(node, args, "div")

    def _op_softmax(self, node, args, kwargs):
        dim = self._arg(node, 1, "dim", -1)
        self._emit(node, OpBuilder.softmax(self._v(args[0]), dim))

    def _op_argmax(self, node, args, kwargs):
        dim = self._arg(node, 1, "dim", None)
        keepdim = self._arg(node, 2, "keepdim", False)
        x = self._v(args[0])
        if dim is None:
            x = self._reshape_value(x, (x.type.numel,))
            dim = 0
        ev = _meta_val(node)
        self._emit(node, OpBuilder.argmax(x, dim, dtype=_DT[ev.dtype] if isinstance(ev, torch.Tensor)
                                          else "int64", keepdim=keepdim))

    def _reduction(self, node, args, kwargs, name):
        dim = self._arg(node, 1, "dim", None)
        keepdim = self._arg(node, 2, "keepdim", False)
        if isinstance(dim, (tuple, list)):
            if len(dim) != 1:
                raise ValueError(f"{name} over several dims is not supported")
            dim = dim[0]
        if dim is None:
            raise ValueError(f"{name} over all elements is not supported")
        self._emit(node, OpBuilder.reduce(name, self._v(args[0]), dim, keepdim))

    def _op_mean(self, node, args, kwargs):
        self._reduction(node, args, kwargs, "mean")

    def _op_sum(self, node, args, kwargs):
        self._reduction(node, args, kwargs, "sum")

    def _op_amax(self, node, args, kwargs):
        self._reduction(node, args, kwargs, "max")

    def _op_layer_norm(self, node, args, kwargs):
        shape = self._arg(node, 1, "normalized_shape")
        if len(shape) != 1:
            raise ValueError("layer_norm over more than the last dim is not supported")
        w = self._arg(node, 2, "weight")
        b = self._arg(node, 3, "bias")
        eps = self._arg(node, 4, "eps", 1e-5)
        self._emit(node, OpBuilder.layer_norm(self._v(args[0]), self._v(w) if w is not None else None,
                                              self._v(b) if b is not None else None, eps))

    def _op_rms_norm(self, node, args, kwargs):
        shape = self._arg(node, 1, "normalized_shape")
        if len(shape) != 1:
            raise ValueError("rms_norm over more than the last dim is not supported")
        w = self._arg(node, 2, "weight")
        eps = self._arg(node, 3, "eps", None)
        if eps is None:
            eps = torch.finfo(_meta_val(node).dtype).eps
        self._emit(node, OpBuilder.rms_norm(self._v(args[0]), self._v(w) if w is not None else None, eps))

    def _op_to(self, node, args, kwargs):
        x = self._v(args[0])
        ev = _meta_val(node)
        dtype = _DT[ev.dtype] if isinstance(ev, torch.Tensor) else x.type.dtype
        if dtype == x.type.dtype:
            self.value_map[node] = x
        else:
            self._emit(node, OpBuilder.to(x, dtype))

    def _reshape_value(self, x: Value, shape) -> Value:
        op = OpBuilder.reshape(x, shape)
        self.fn.block.add_op(op)
        return op.outputs[0]

    def _op_reshape(self, node, args, kwargs):
        x = self._v(args[0])
        shape = self._ex_shape(node)
        if shape == x.type.shape:
            self.value_map[node] = x
        else:
            self._emit(node, OpBuilder.reshape(x, shape))

    def _op_permute(self, node, args, kwargs):
        dims = args[1:] if len(args) > 2 else (args[1] if len(args) > 1 else kwargs["dims"])
        self._emit(node, OpBuilder.transpose(self._v(args[0]), tuple(dims)))

    def _op_transpose(self, node, args, kwargs):
        x = self._v(args[0])
        if len(args) == 1:  # .t()
            d0, d1 = 0, 1
        else:
            d0, d1 = args[1], args[2]
        rank = len(x.type.shape)
        perm = list(range(rank))
        d0, d1 = d0 % rank, d1 % rank
        perm[d0], perm[d1] = perm[d1], perm[d0]
        self._emit(node, OpBuilder.transpose(x, tuple(perm)))

    def _op_interpolate(self, node, args, kwargs):
        mode = kwargs.get("mode", args[3] if len(args) > 3 else "nearest")
        ac = kwargs.get("align_corners", args[4] if len(args) > 4 else None)
        if mode != "bilinear" or ac:
            raise ValueError(f"interpolate: only bilinear with align_corners=False is supported (got {mode}, "
                             f"{ac})")
        if kwargs.get("antialias", False):
            raise ValueError("interpolate: antialias is not supported")
        shape = self._ex_shape(node)
        x = self._v(args[0])
        layout = "NCHW" if len(shape) == 4 else "CHW"
        self._emit(node, OpBuilder.resize(x, (shape[-2], shape[-1]), layout=layout))

    def _op_conv2d(self, node, args, kwargs):
        """Patchify convolution (stride == kernel, no padding) as reshape → permute → linear."""
        self._patchify(node, self._arg(node, 1, "weight"), self._arg(node, 2, "bias"), self._arg(node, 3, "stride", 1),
                       self._arg(node, 4, "padding", 0), self._arg(node, 5, "dilation", 1),
                       self._arg(node, 6, "groups", 1))

    def _patchify(self, node, w_node, b_node, stride, padding, dilation, groups):
        x = self._v(node.args[0])
        w = self._v(w_node)
        O, C, kh, kw = w.type.shape
        st = tuple(stride) if isinstance(stride, (tuple, list)) else (stride, stride)
        pd = tuple(padding) if isinstance(padding, (tuple, list)) else (padding, padding)
        dl = tuple(dilation) if isinstance(dilation, (tuple, list)) else (dilation, dilation)
        if st != (kh, kw) or pd != (0, 0) or dl != (1, 1) or groups != 1:
            raise ValueError("conv2d: only non-overlapping patchify convolutions are supported")
        B, Cx, H, W = x.type.shape
        if H % kh or W % kw:
            raise ValueError("conv2d: image size must be a multiple of the patch size")
        gh, gw = H // kh, W // kw
        r = self._reshape_value(x, (B, C, gh, kh, gw, kw))
        tp = OpBuilder.transpose(r, (0, 2, 4, 1, 3, 5))
        self.fn.block.add_op(tp)
        flat = self._reshape_value(tp.outputs[0], (B * gh * gw, C * kh * kw))
        w2 = self._reshape_value(w, (O, C * kh * kw))
        lin = OpBuilder.linear(flat, w2, self._v(b_node) if b_node is not None else None)
        self.fn.block.add_op(lin)
        y = self._reshape_value(lin.outputs[0], (B, gh, gw, O))
        self._emit(node, OpBuilder.transpose(y, (0, 3, 1, 2)))

    def _op_narrow(self, node, args, kwargs):
        x = self._v(args[0])
        dim, start, length = self._arg(node, 1, "dim"), self._arg(node, 2, "start"), self._arg(node, 3, "length")
        self._emit(node, OpBuilder.slice(x, dim, start, start + length))

    def _slices(self, node, x: Value, dim: int, sizes) -> None:
        outs, pos = [], 0
        for n in sizes:
            op = OpBuilder.slice(x, dim, pos, pos + n)
            self.fn.block.add_op(op)
            outs.append(op.outputs[0])
            pos += n
        self.tuple_map[node] = outs

    def _op_chunk(self, node, args, kwargs):
        x = self._v(args[0])
        chunks, dim = self._arg(node, 1, "chunks"), self._arg(node, 2, "dim", 0)
        size = x.type.shape[dim]
        step = -(-size // chunks)
        self._slices(node, x, dim, [min(step, size - i) for i in range(0, size, step)])

    def _op_split(self, node, args, kwargs):
        x = self._v(args[0])
        sz, dim = self._arg(node, 1, "split_size_or_sections", self._arg(node, 1, "split_size")), \
            self._arg(node, 2, "dim", 0)
        size = x.type.shape[dim]
        if isinstance(sz, int):
            sizes = [min(sz, size - i) for i in range(0, size, sz)]
        else:
            sizes = list(sz)
        self._slices(node, x, dim, sizes)

    def _op_cat(self, node, args, kwargs):
        xs = self._arg(node, 0, "tensors")
        dim = self._arg(node, 1, "dim", 0)
        self._emit(node, OpBuilder.cat([self._v(t) for t in xs], dim))

    def _op_expand(self, node, args, kwargs):
        x = self._v(args[0])
        self._emit(node, OpBuilder.expand(x, self._ex_shape(node)))

    def _op_rope(self, node, args, kwargs):
        x, c, s_ = (self._v(a) for a in args[:3])
        self._emit(node, OpBuilder.rope(x, c, s_))

    def _op_sdpa(self, node, args, kwargs):
        q, k, v = (self._v(a) for a in args[:3])
        if self._arg(node, 3, "attn_mask") is not None:
            raise ValueError("scaled_dot_product_attention with a mask is not supported")
        if self._arg(node, 4, "dropout_p", 0.0):
            raise ValueError("scaled_dot_product_attention with dropout is not supported")
        self._emit(node, OpBuilder.sdpa(q, k, v, self._arg(node, 6, "scale"), self._arg(node, 5, "is_causal", False)))
