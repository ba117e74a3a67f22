"""torch.export importer: ``ExportedProgram`` → DevProc IR Function.

The reference's design documents name ``torch.export`` output as the model
entry point (CLAUDE.md:9) and plan a ``TorchExportImporter`` that turns an
``ExportedProgram`` into IR ops, with the weights and biases recorded as
constant tensors (docs/MVP实施计划.md:146-185); its source tree never
implemented it (the FX path, src/devproc/ir/from_torch.py:87-140, captures
with Dynamo instead).

An exported graph is an FX graph over ATen overloads (``aten.linear.default``,
``aten.add.Tensor``, …) whose placeholders are, in order, the lifted
parameters, buffers and tensor constants, then the user inputs; the graph
signature says which is which.  The importer reuses the FX converter's op
handlers (the overload's packet name is the handler key) and adds the ATen
forms the Dynamo graph does not have: ``embedding(weight, indices)``,
``select.int``, ``slice.Tensor``, ``upsample_bilinear2d.vec``,
``_to_copy``, ``dropout`` in eval mode, and the metadata asserts (dropped).
Graphs lowered to core ATen (``ep.run_decompositions()``) import too for
``addmm`` (a linear when its right operand is a transposed weight),
``native_layer_norm`` (its normalised output), ``_softmax``, patchify
``convolution`` and ``_unsafe_view``; the math form of attention that
decomposition produces (with boolean guards for fully masked rows) does not:
export without decompositions keeps ``scaled_dot_product_attention`` whole.
Lifted parameters, buffers and constants become ``fn.constants``, so the
compiled program uploads them once; only the user inputs stay run-time
inputs, named after the exported function's arguments.
"""

import operator
from typing import Any, Dict, Optional

import torch
import torch.fx

from .function import Function
from .fx_converter import FXToIRConverter, _meta_val
from .ops import OpBuilder

_CONST_KINDS = ("PARAMETER", "BUFFER", "CONSTANT_TENSOR")
# ATen calls with no tensor result that only check metadata at trace time.
_DROPPED = {"_assert_tensor_metadata", "_assert_scalar", "sym_constrain_range_for_size",
            "sym_constrain_range", "_assert_async"}


class TorchExportImporter(FXToIRConverter):
    """``TorchExportImporter().import_program(ep)`` → IR Function with the
    program's parameters, buffers and lifted constants as ``fn.constants``."""

    def import_program(self, ep: "torch.export.ExportedProgram") -> Function:
        sig = ep.graph_signature
        for out in sig.output_specs:
            if out.kind.name != "USER_OUTPUT":
                raise ValueError(f"exported program mutates state ({out.kind.name} {out.target}); "
                                 "DevProc programs are pure functions")
        self._consts: Dict[str, torch.Tensor] = {}
        self._user = set()
        for spec in sig.input_specs:
            kind = spec.kind.name
            name = spec.arg.name
            if kind in _CONST_KINDS:
                t = ep.state_dict.get(spec.target) if spec.target in ep.state_dict else \
                    ep.constants.get(spec.target)
                if not isinstance(t, torch.Tensor):
                    raise ValueError(f"exported {kind.lower()} {spec.target} has no tensor value")
                self._consts[name] = t
            elif kind == "USER_INPUT":
                self._user.add(name)
            else:
                raise ValueError(f"unsupported exported input kind {kind} ({name})")
        fn = self.convert(ep.graph_module, ())
        fn._name = "exported_program"
        return fn

    # Alias matching the planned importer's verb.
    convert_program = import_program

    # ------------------------------------------------------------- nodes
    def _on_placeholder(self, node) -> None:
        if node.name in self._consts:
            t = self._consts[node.name]
            self._add_input(node, node.name, t, True)
            return
        if node.name not in self._user:
            raise ValueError(f"placeholder {node.name} is not in the graph signature")
        ev = _meta_val(node)
        if not isinstance(ev, torch.Tensor):
            raise ValueError(f"user input {node.name} is not a tensor")
        self._add_input(node, node.name, ev, False)

    def _on_call_function(self, node) -> None:
        t = node.target
        if isinstance(t, torch._ops.OpOverload):
            if t.overloadpacket.__name__ in _DROPPED:
                return
            if t._schema.is_mutable:  # in-place ATen op (training-IR exports keep them)
                raise ValueError(f"exported program mutates state ({t}); DevProc programs are pure functions")
        super()._on_call_function(node)

    def _dispatch(self, node, name: str, args, kwargs) -> None:
        special = getattr(self, "_aten_" + name, None)
        if special is not None:
            return special(node, args, kwargs)
        super()._dispatch(node, name, args, kwargs)

    # ----------------------------------------------------- ATen-only forms
    def _aten_embedding(self, node, args, kwargs):
        """aten.embedding(weight, indices, padding_idx, scale_grad, sparse)."""
        self._emit(node, OpBuilder.embedding(self._v(args[1]), self._v(args[0])))

    def _aten_select(self, node, args, kwargs):
        """aten.select.int(x, dim, index): a one-element slice with the dim dropped."""
        x = self._v(args[0])
        dim = args[1] % len(x.type.shape)
        size = x.type.shape[dim]
        i = args[2] + size if args[2] < 0 else args[2]
        if not 0 <= i < size:
            raise ValueError(f"select {node.name}: index {args[2]} out of range")
        op = OpBuilder.slice(x, dim, i, i + 1)
        self.fn.block.add_op(op)
        self.value_map[node] = self._reshape_value(op.outputs[0], self._ex_shape(node))

    def _aten_slice(self, node, args, kwargs):
        """aten.slice.Tensor(x, dim=0, start=None, end=None, step=1); ends clamp like Python slices."""
        x = self._v(args[0])
        dim = self._arg(node, 1, "dim", 0) % len(x.type.shape)
        size = x.type.shape[dim]
        start = self._arg(node, 2, "start", None)
        end = self._arg(node, 3, "end", None)
        step = self._arg(node, 4, "step", 1)
        start, end, step = slice(start, end, step).indices(size)
        if (start, end, step) == (0, size, 1):
            self.value_map[node] = x
            return
        self._emit(node, OpBuilder.slice(x, dim, start, end, step))

    def _aten_upsample_bilinear2d(self, node, args, kwargs):
        """aten.upsample_bilinear2d.vec(x, output_size, align_corners, scale_factors)."""
        if self._arg(node, 2, "align_corners", False):
            raise ValueError("upsample_bilinear2d: only align_corners=False is supported")
        shape = self._ex_shape(node)
        layout = "NCHW" if len(shape) == 4 else "CHW"
        self._emit(node, OpBuilder.resize(self._v(args[0]), (shape[-2], shape[-1]), layout=layout))

    # -------------------------------------- core-ATen forms (run_decompositions)
    def _aten_addmm(self, node, args, kwargs):
        """aten.addmm(bias, x, w.t()) → linear(x, w, bias) when the right operand
        is the transpose of a weight [N, K]; else matmul + add."""
        if self._arg(node, 3, "beta", 1) != 1 or self._arg(node, 4, "alpha", 1) != 1:
            raise ValueError("addmm with beta or alpha other than 1 is not supported")
        bias, x, m2 = args[0], args[1], args[2]
        src = self._transposed_source(m2)
        if src is not None:
            self._emit(node, OpBuilder.linear(self._v(x), self._v(src), self._v(bias)))
            return
        mm = OpBuilder.matmul(self._v(x), self._v(m2), out_dtype=self._v(x).type.dtype)
        self.fn.block.add_op(mm)
        self._emit(node, OpBuilder.binary("add", mm.outputs[0], self._v(bias)))

    @staticmethod
    def _transposed_source(n):
        """The [N, K] node that ``n`` transposes (aten.t / permute [1, 0]), if any."""
        if not isinstance(n, torch.fx.Node) or n.op != "call_function":
            return None
        t = n.target
        name = t.overloadpacket.__name__ if isinstance(t, torch._ops.OpOverload) else ""
        if name == "t" or (name == "permute" and list(n.args[1]) == [1, 0]) or \
                (name == "transpose" and sorted(a % 2 for a in n.args[1:3]) == [0, 1]):
            return n.args[0]
        return None

    def _aten_native_layer_norm(self, node, args, kwargs):
        """aten.native_layer_norm(x, shape, w, b, eps) → (out, mean, rstd); only out is used."""
        shape = args[1]
        if len(shape) != 1:
            raise ValueError("layer_norm over more than the last dim is not supported")
        w, b, eps = args[2], args[3], args[4]
        op = OpBuilder.layer_norm(self._v(args[0]), self._v(w) if w is not None else None,
                                  self._v(b) if b is not None else None, eps)
        self.fn.block.add_op(op)
        self.tuple_map[node] = [op.outputs[0], None, None]
        for user in node.users:
            if not (user.target is operator.getitem and user.args[1] == 0):
                raise ValueError("native_layer_norm: only the normalised output may be used")

    def _aten__softmax(self, node, args, kwargs):
        """aten._softmax(x, dim, half_to_float).  With half_to_float a 16-bit
        input gives an fp32 result: the input is cast to fp32 first (the
        softmax itself runs in fp32 either way)."""
        x = self._v(args[0])
        half_to_float = len(args) > 2 and bool(args[2])
        if half_to_float and x.type.dtype in ("float16", "bfloat16"):
            cast = OpBuilder.to(x, "float32")
            self.fn.block.add_op(cast)
            x = cast.outputs[0]
        self._emit(node, OpBuilder.softmax(x, args[1]))

    def _aten_convolution(self, node, args, kwargs):
        """aten.convolution(x, w, b, stride, padding, dilation, transposed, output_padding, groups)."""
        if args[6] or any(args[7]):
            raise ValueError("transposed convolution is not supported")
        self._patchify(node, args[1], args[2], args[3], args[4], args[5], args[8])

    def _aten__unsafe_view(self, node, args, kwargs):
        self._op_reshape(node, args, kwargs)

    def _aten__to_copy(self, node, args, kwargs):
        self._op_to(node, args, kwargs)

    def _aten_dropout(self, node, args, kwargs):
        if self._arg(node, 2, "train", False):
            raise ValueError("dropout in training mode is not supported")
        self.value_map[node] = self._v(args[0])

    def _aten_alias(self, node, args, kwargs):
        self.value_map[node] = self._v(args[0])

    _aten_lift_fresh_copy = _aten_alias


def import_exported_program(ep: "torch.export.ExportedProgram") -> Function:
    """IR Function of an ``ExportedProgram`` (parameters and buffers as constants)."""
    return TorchExportImporter().import_program(ep)


def is_exported_program(obj: Any) -> bool:
    return isinstance(obj, torch.export.ExportedProgram)


def export_module(target, *example_inputs, strict: Optional[bool] = None) -> "torch.export.ExportedProgram":
    """``torch.export.export`` of a module (or a function wrapped in one) under ``no_grad``."""
    if not isinstance(target, torch.nn.Module):
        fn = target

        class _Wrap(torch.nn.Module):
            def forward(self, *a):
                return fn(*a)

        target = _Wrap()
    kw = {} if strict is None else {"strict": strict}
    with torch.no_grad():
        return torch.export.export(target, tuple(example_inputs), **kw)
