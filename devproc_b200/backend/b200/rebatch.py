"""Batch separability: is a program the same computation on each sample, and
its copy for a smaller batch.

The reference's ``run`` copied every input to the device, ran all ops and
copied the outputs back one after another (src/devproc/backend/triton/
compiler.py:189-250).  For a program whose samples are independent, the
runtime can instead run it on chunks of the batch while the next chunk's
input crosses PCIe and the previous chunk's output comes back, so the
transfers overlap each other and the kernels.  That needs two things, both
decided here on the IR at compile time:

* ``batch_factors(fn)`` proves independence: every run-time input has the
  same leading dim B, every output is batched, and each op maps samples to
  samples.  A batched value's leading dim is B·f, with sample i owning rows
  [i·f, (i+1)·f) — so a ``reshape`` of [B, L, D] to [B·L, D] stays batched
  (f = L) and a ``linear`` over its rows too, while a reduction or slice
  along dim 0, a cat along dim 0 or a broadcast across samples is not.
  Constants and values computed only from constants are shared by all
  samples.
* ``rebatch(fn, b)`` rebuilds the function for batch b: every batched type's
  leading dim becomes b·f (and the shape attribute of reshape / expand with
  it); everything else is copied.
"""

from typing import Dict, Optional, Tuple

from ...ir.base import Op, Value
from ...ir.function import Function
from ...ir.types import TensorType

_UNARY = {"relu", "sigmoid", "tanh", "exp", "neg", "abs", "silu", "gelu", "to",
          "add_scalar", "sub_scalar", "mul_scalar", "div_scalar", "pow_scalar"}
_BINARY = {"add", "sub", "mul", "div"}
_LASTDIM_ROW = {"layer_norm", "rms_norm"}
_DIM_ROW = {"softmax", "argmax", "sum", "max", "min", "mean"}


def _shape(v: Value) -> Tuple[int, ...]:
    return tuple(v.type.shape) if isinstance(v.type, TensorType) else ()


def _broadcasts_past_batch(shared: Value, out_rank: int) -> bool:
    """A shared (unbatched) operand broadcast to a batched result must not
    span the batch dim: fewer dims, or size 1 where dim 0 lines up."""
    s = _shape(shared)
    lead = out_rank - len(s)
    return lead > 0 or (lead == 0 and s[0] == 1)


class _Why(Exception):
    pass


def _out_factor(op: Op, fac: Dict[str, int], B: int) -> Optional[int]:
    """Batch factor of ``op``'s result, None when it is shared; raises _Why
    when the op mixes samples."""
    ins = op.inputs
    facs = [fac.get(v.name) for v in ins]
    if all(f is None for f in facs):
        return None
    name = op.name
    out = op.outputs[0]
    oshape = _shape(out)
    x, fx = ins[0], facs[0]
    xshape = _shape(x)

    def need(cond, why):
        if not cond:
            raise _Why(f"{name}: {why}")

    if name in _UNARY:
        need(fx is not None, "batched operand expected first")
        return fx
    if name == "normalize":
        need(fx is not None and op.attr("channel_dim", 1) != 0, "channels along the batch dim")
        return fx
    if name in _BINARY:
        bf = {f for f in facs if f is not None}
        need(len(bf) == 1, "operands batched differently")
        f = bf.pop()
        for v, fv in zip(ins, facs):
            if fv is None:
                need(_broadcasts_past_batch(v, len(oshape)), "shared operand spans the batch dim")
            else:
                need(len(_shape(v)) == len(oshape) and _shape(v)[0] == oshape[0], "batched operand broadcast")
        return f
    if name in _DIM_ROW:
        need(fx is not None and len(xshape) >= 2, "reduction of a 1-d batched value")
        need(op.attr("dim", -1) % len(xshape) != 0, "reduction along the batch dim")
        return fx
    if name in _LASTDIM_ROW:
        need(fx is not None and len(xshape) >= 2, "norm of a 1-d batched value")
        need(all(f is None for f in facs[1:]), "batched norm weights")
        return fx
    if name == "resize":
        need(fx is not None and str(op.attr("layout", "")).startswith("N"), "resize without a batch dim")
        return fx
    if name == "transpose":
        need(fx is not None and tuple(op.attr("dims"))[0] == 0, "transpose moves the batch dim")
        return fx
    if name == "reshape":
        need(fx is not None and len(oshape) >= 1 and oshape[0] >= B and oshape[0] % B == 0,
             "reshape splits or merges across samples")
        return oshape[0] // B
    if name == "slice":
        need(fx is not None and op.attr("dim") % len(xshape) != 0, "slice along the batch dim")
        return fx
    if name == "expand":
        need(fx is not None and len(oshape) == len(xshape) and oshape[0] == xshape[0], "expand across samples")
        return fx
    if name == "cat":
        need(all(f is not None and f == fx for f in facs), "cat of batched and shared values")
        need(op.attr("dim") % len(oshape) != 0, "cat along the batch dim")
        return fx
    if name == "rope":
        need(fx is not None, "rope of a shared value")
        for v, fv in zip(ins[1:], facs[1:]):
            if fv is None:
                need(_broadcasts_past_batch(v, len(xshape)), "rotary table spans the batch dim")
            else:
                need(fv == fx and _shape(v)[0] == xshape[0], "rotary table batched differently")
        return fx
    if name == "linear":
        need(fx is not None and len(xshape) >= 2, "linear of a 1-d batched value")
        need(all(f is None for f in facs[1:]), "batched weights")
        return fx
    if name == "matmul":
        fb = facs[1]
        if fb is None:
            need(fx is not None and len(xshape) >= 2 and len(_shape(ins[1])) == 2, "matmul broadcast")
            return fx
        need(fx == fb and len(xshape) >= 3 and len(_shape(ins[1])) == len(xshape), "batched matmul shapes")
        return fx
    if name == "embedding":
        need(fx is not None and facs[1] is None, "batched embedding table")
        return fx
    if name == "sdpa":
        need(all(f == fx for f in facs) and fx is not None and len(xshape) >= 3, "attention across samples")
        return fx
    raise _Why(f"{name}: not known to be per-sample")


def batch_factors(fn: Function, constants=()) -> Tuple[Optional[int], Dict[str, int], str]:
    """(B, {value name: factor}, "") when ``fn`` is batch-separable, else
    (None, {}, reason)."""
    consts = set(constants) | set(getattr(fn, "constants", {}) or {})
    runtime = [v for v in fn.inputs if v.name not in consts]
    if not runtime:
        return None, {}, "no run-time inputs"
    shapes = [_shape(v) for v in runtime]
    if any(len(s) == 0 for s in shapes):
        return None, {}, "scalar input"
    B = shapes[0][0]
    if B < 2 or any(s[0] != B for s in shapes):
        return None, {}, "inputs do not share a leading batch dim"
    fac = {v.name: 1 for v in runtime}
    try:
        for op in fn.block.ops:
            if op.name in ("input", "return"):
                continue
            if len(op.outputs) != 1 or not isinstance(op.outputs[0].type, TensorType):
                raise _Why(f"{op.name}: not a single tensor result")
            f = _out_factor(op, fac, B)
            if f is not None:
                fac[op.outputs[0].name] = f
    except _Why as e:
        return None, {}, str(e)
    if not fn.outputs or any(o.name not in fac for o in fn.outputs):
        return None, {}, "an output is shared by all samples"
    return B, fac, ""


def rebatch(fn: Function, b: int, constants=()) -> Function:
    """Copy of ``fn`` for batch ``b`` (``fn`` must be batch-separable)."""
    B, fac, why = batch_factors(fn, constants)
    if B is None:
        raise ValueError(f"program is not batch-separable: {why}")
    new: Dict[str, Value] = {}

    def retype(v: Value) -> TensorType:
        t = v.type
        if v.name not in fac:
            return t
        return TensorType((b * fac[v.name],) + tuple(t.shape[1:]), t.dtype, t.device)

    out_fn = Function(f"{fn.name}_b{b}")
    out_fn.constants = dict(getattr(fn, "constants", {}) or {})
    for v in fn.inputs:
        nv = Value(v.name, retype(v))
        new[v.name] = nv
        out_fn.add_input(nv)
    for op in fn.block.ops:
        if op.name in ("input", "return"):
            continue
        outs = [Value(o.name, retype(o)) for o in op.outputs]
        attrs = dict(op.attrs)
        if op.name in ("reshape", "expand") and op.outputs[0].name in fac:
            attrs["shape"] = tuple(outs[0].type.shape)
        nop = Op(op.name, [new[i.name] for i in op.inputs], outs, attrs)
        out_fn.block.add_op(nop)
        for o in outs:
            new[o.name] = o
    out_fn.outputs = [new[o.name] for o in fn.outputs]
    return out_fn
