"""Lower an IR Function to launch records over a statically planned arena.

Replaces the reference's compile step (src/devproc/backend/triton/
compiler.py:476-536), which recorded ``tensor_allocations`` and placeholder
kernel specs and left all real work to a per-call, per-op JIT loop
(compiler.py:206-358).  Here every decision is made once, on the host, at
compile time:

* fusion — one launch per dataflow region:
    - ``resize`` → [to(f32)] → [normalize] → [transpose to planar] → [to(float)]
      becomes one preprocessing record (``dp_preproc``);
    - ``linear``/``matmul`` absorb a following bias add, one activation
      (relu / gelu / silu), a residual add and a float cast into the GEMM
      epilogue (``dp_gemm``);
    - softmax / argmax / sum / max / min / mean / layer_norm / rms_norm over the
      last dim become one row-reduction record, argmax absorbing its int cast;
    - remaining chains of elementwise ops (casts, normalise, activations,
      broadcast arithmetic, transposes) become one region record each;
* views — ``reshape`` aliases storage, ``transpose`` only permutes strides;
  a consumer that needs contiguous data gets a region copy;
* memory — every intermediate lives in one arena at an offset chosen by
  liveness (first fit, 256-byte aligned), so running allocates nothing.
"""

import ctypes
import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

from ... import _native as N
from ...ir.base import Op, Value
from ...ir.function import Function
from ...ir.types import DTYPE_BYTES, FLOAT_DTYPES, ScalarType, TensorType
from ..base import CompilationError, UnsupportedOpError

ALIGN = 256

ELEMENTWISE_UNARY = {"relu": "relu", "sigmoid": "sigmoid", "tanh": "tanh", "exp": "exp", "neg": "neg",
                     "abs": "abs", "silu": "silu"}
ELEMENTWISE_BINARY = {"add": "add", "sub": "sub", "mul": "mul", "div": "div"}
SCALAR_OPS = {"add_scalar": "add", "sub_scalar": "sub", "mul_scalar": "mul", "div_scalar": "div",
              "pow_scalar": None}
ELEMENTWISE = (set(ELEMENTWISE_UNARY) | set(ELEMENTWISE_BINARY) | {k for k, v in SCALAR_OPS.items() if v}
               | {"gelu", "to", "normalize", "transpose", "reshape"})
ROW_OPS = {"softmax", "argmax", "sum", "max", "min", "mean", "layer_norm", "rms_norm"}
HOST_OPS = {"load_tokenizer", "tokenize_encode", "tokenize_decode", "string_length", "string_concat",
            "string_slice", "string_format", "dict_create", "dict_get", "dict_set", "dict_size"}


def contiguous_strides(shape: Tuple[int, ...]) -> Tuple[int, ...]:
    st, acc = [], 1
    for s in reversed(shape):
        st.append(acc)
        acc *= s
    return tuple(reversed(st))


def view_reshape(shape, strides, new_shape):
    """Strides that present (shape, strides) as ``new_shape`` without copying, or None.

    Dims that are laid out back to back (stride[i] == stride[i+1] * shape[i+1])
    form runs that behave like one dim; every new dim must fall inside one run.
    """
    runs = []  # (size, innermost stride), outermost first
    for sz, st in zip(shape, strides):
        if sz == 1:
            continue
        if runs and runs[-1][1] == st * sz:
            runs[-1] = (runs[-1][0] * sz, st)
        else:
            runs.append((sz, st))
    out = [0] * len(new_shape)
    ri = len(runs) - 1
    left, unit = (runs[ri][0], runs[ri][1]) if runs else (1, 1)
    for i in range(len(new_shape) - 1, -1, -1):
        n = new_shape[i]
        if n == 1:
            out[i] = 0
            continue
        while left == 1 and ri > 0:
            ri -= 1
            left, unit = runs[ri]
        if left % n != 0:
            return None
        out[i] = unit
        unit *= n
        left //= n
    if left != 1 or ri > 0:
        return None
    return tuple(out)


def _prod(xs) -> int:
    p = 1
    for x in xs:
        p *= x
    return p


@dataclass(eq=False)
class Buffer:
    """One storage slot of the program."""
    kind: str            # "input" | "const" | "output" | "arena"
    dtype: str
    shape: Tuple[int, ...]
    name: str
    offset: int = 0      # arena byte offset
    first: int = -1      # first record touching it
    last: int = -1       # last record touching it
    slot: int = -1
    base: Optional["Buffer"] = None  # set for a slot naming a sub-range of another buffer
    base_off: int = 0                # byte offset of that sub-range

    @property
    def nbytes(self) -> int:
        return max(1, _prod(self.shape)) * DTYPE_BYTES[self.dtype]

    @property
    def root(self) -> "Buffer":
        return self.base if self.base is not None else self


@dataclass
class View:
    """An IR value seen as (buffer, shape, element strides, element offset)."""
    buf: Buffer
    shape: Tuple[int, ...]
    strides: Tuple[int, ...]
    offset: int = 0

    @property
    def contiguous(self) -> bool:
        return self.offset == 0 and all(
            st == cs for st, cs, s in zip(self.strides, contiguous_strides(self.shape), self.shape) if s != 1)


@dataclass
class Record:
    kernel: int
    operands: List[Optional[Buffer]]
    params: ctypes.Structure
    label: str
    flops: int = 0
    bytes: int = 0


@dataclass
class Lowered:
    """Everything the runtime needs: buffers, records, I/O order."""
    name: str
    buffers: List[Buffer]
    records: List[Record]
    inputs: List[Tuple[str, Buffer]]          # runtime inputs in IR order
    consts: List[Tuple[str, Buffer]]          # inputs bound once from constants
    outputs: List[Tuple[str, Buffer]]         # function outputs in order
    arena_bytes: int = 0
    labels: List[str] = field(default_factory=list)
    extra_consts: Dict[str, "torch.Tensor"] = field(default_factory=dict)  # constants made by the lowering

    @property
    def aliases(self) -> List[Tuple[int, int, int]]:
        """(slot, root slot, byte offset) of every caller-bound sub-range slot."""
        return [(b.slot, b.root.slot, b.base_off) for b in self.buffers
                if b.base is not None and b.root.kind != "arena"]

    def plan_bytes(self) -> bytes:
        """Serialise to the dp_plan blob (header, slots, records)."""
        hdr = N.PlanHeader(N.DP_PLAN_MAGIC, N.DP_PLAN_VERSION, len(self.buffers), len(self.records),
                           self.arena_bytes, 0)
        out = [bytes(hdr)]
        for b in self.buffers:
            arena = b.root.kind == "arena"
            kind = N.DP_SLOT_ARENA if arena else N.DP_SLOT_BOUND
            out.append(bytes(N.PlanSlot(kind, N.DTYPE_CODE[b.dtype], b.offset if arena else 0, b.nbytes)))
        for r in self.records:
            rec = N.PlanRecord()
            rec.kernel = r.kernel
            rec.n_operands = len(r.operands)
            for i in range(N.DP_RECORD_MAX_OPERANDS):
                rec.operand[i] = -1
            for i, b in enumerate(r.operands):
                rec.operand[i] = b.slot if b is not None else -1
            raw = bytes(r.params)
            ctypes.memmove(rec.params, raw, len(raw))
            out.append(bytes(rec))
        return b"".join(out)


# ------------------------------------------------------------- split-K
_SMS = 148  # B200


def splitk_factor(M: int, N: int, K: int, tf32: bool, b_layout: int) -> int:
    """Number of K slices for a tensor-core GEMM, 1 = no split.

    Tiles: 256 x 256 on CTA pairs (74 per GPU) when M and N exceed one CTA's
    share, else 128 x 256 on single CTAs; a stage covers 128 bf16 or 64 TF32
    K.  A GEMM with fewer tiles than half the pairs and at least 8 stages is
    split when the modelled time - waves x (stages per slice + 3 for pipeline
    fill and epilogue) at 1 us per stage, plus 3 us and the workspace traffic
    at 5 TB/s for the reduction - drops by 10 % or more.  Slices are whole
    stages (S divides the stage count) so every slice's K is the same.
    """
    cg = 2 if (M > 128 and N > 128) else 1
    pairs = _SMS // cg
    tiles = -(-M // (128 * cg)) * -(-N // 256)
    box_k = 32 if tf32 else 64
    kstep = box_k * (2 if cg == 2 else 1)
    if K % kstep or tiles * 2 > pairs:
        return 1
    kb = K // kstep
    if kb < 8:
        return 1

    def cost(S):
        t = -(-tiles * S // pairs) * (kb / S + 3.0)
        return t + (3.0 + (S + 1) * M * N * 4 / 5e6 if S > 1 else 0.0)

    best, best_s = cost(1), 1
    for S in range(2, 17):
        if kb % S == 0 and cost(S) < best:
            best, best_s = cost(S), S
    return best_s if best <= 0.9 * cost(1) else 1


def streamk_bytes(M: int, n: int, K: int, batch: int, tf32: bool, epilogue: int) -> int:
    """Workspace bytes of a stream-K tensor-core GEMM, 0 = whole tiles.

    Same plan as the kernel's launcher (for 148 SMs; the launcher re-plans
    for the device it runs on and uses whole tiles if the plan changes):
    the tiles past the last full wave (``rem``, with ``waves`` full waves of
    CTA groups) are split by K stage when each group's even share of their
    stages is at least half a tile (at most three runs per tile) and waves x
    stages + the share + 2 + 1.5 per partial handed on is at most 0.9 of the
    whole-tile time, (waves + 1) x stages.  The workspace is the per-tile counters
    plus one 128 KB fp32 partial slot per SM (the C-ABI's bound).
    """
    if epilogue & (N.DP_EPI_SOFTMAX | N.DP_EPI_ARGMAX):
        return 0
    cg = 2 if (M > 128 and n > 128) else 1
    groups = _SMS // cg
    tiles = -(-M // (128 * cg)) * -(-n // 256) * batch
    kb = -(-K // ((32 if tf32 else 64) * (2 if cg == 2 else 1)))
    rem, waves = tiles % groups, tiles // groups
    if rem == 0 or kb < 4:
        return 0
    ipp = -(-rem * kb // groups)
    if 2 * ipp < kb:
        return 0
    runs = -(-kb // ipp) + 1
    if waves * kb + ipp + 2.0 + 1.5 * (runs - 1) > 0.9 * (waves + 1) * kb:
        return 0
    counters = -(-4 * -(-M // 128) * -(-n // 256) * batch // 256) * 256
    return counters + _SMS * 64 * 128 * 16


class Lowerer:
    use_fused_attention = True  # bf16 sdpa as one fused tensor-core kernel (else GEMM + softmax + GEMM)
    # GEMMs with a ragged last wave split it by K stage.  Off by default: on
    # B200 the split runs' hand-off (partial write, wait, read back, a second
    # epilogue) costs more than the idle CTA pairs it fills - 3,200 x 1,024,
    # K 4,096 runs 41.0 us split against 36.4 us with whole tiles.
    use_streamk = False

    def __init__(self, fn: Function, const_names=(), const_tensors=None):
        self.fn = fn
        self.const_names = set(const_names)
        self.const_tensors = dict(const_tensors or {})
        self.new_consts: List[Tuple[str, Buffer]] = []
        self.views: Dict[str, View] = {}
        # values whose producer wrote them directly as a 3xTF32 operand [hi | hi | lo]
        self.tf32_split_views: Dict[str, View] = {}
        # cat buffers by (dim, shape, dtype, first input): the last cat's view, output and inputs
        self.cat_reuse: Dict[tuple, tuple] = {}
        self.op_index = {id(o): i for i, o in enumerate(fn.block.ops)}
        self.buffers: List[Buffer] = []
        self.records: List[Record] = []
        self.done = set()   # ids of ops already lowered (fused)
        self.uses: Dict[str, List[Op]] = {}
        self.producer: Dict[str, Op] = {}
        self.out_names = {v.name for v in fn.outputs}
        for op in fn.block.ops:
            for v in op.inputs:
                self.uses.setdefault(v.name, []).append(op)
            for v in op.outputs:
                self.producer[v.name] = op

    # ------------------------------------------------------------ helpers
    def new_buffer(self, kind, dtype, shape, name) -> Buffer:
        b = Buffer(kind, dtype, tuple(shape), name)
        self.buffers.append(b)
        return b

    def new_value_view(self, value: Value, dtype=None, shape=None) -> View:
        t = value.type
        shape = tuple(shape if shape is not None else materialized_shape(value))
        dtype = dtype or t.dtype
        buf = self.new_buffer("arena", dtype, shape, value.name)
        v = View(buf, shape, contiguous_strides(shape))
        self.views[value.name] = v
        return v

    def ready(self, v: Value) -> bool:
        """Whether ``v`` has a view now; a pending reshape / transpose producing it
        (a pure view, free to lower early) is lowered here if its input is ready."""
        if v.name in self.views:
            return True
        op = self.producer.get(v.name)
        if op is None or id(op) in self.done or op.name not in ("reshape", "transpose"):
            return False
        if not self.ready(op.inputs[0]):
            return False
        self.lower_op(op)
        self.done.add(id(op))
        return v.name in self.views

    def single_use(self, v: Value) -> Optional[Op]:
        """The only consumer of ``v`` if it has exactly one and is not a function output."""
        us = self.uses.get(v.name, [])
        if len(us) == 1 and v.name not in self.out_names:
            return us[0]
        return None

    def derived_const(self, name: str, dtype: str, shape) -> Buffer:
        """The one slot of a constant the lowering derives (a concatenated or
        padded weight), shared by every record that reads it."""
        for n, b in self.new_consts:
            if n == name:
                return b
        buf = self.new_buffer("const", dtype, tuple(shape), name)
        self.new_consts.append((name, buf))
        return buf

    def alias(self, buf: Buffer, byte_off: int, name: str) -> Buffer:
        """A slot for the bytes of ``buf`` from ``byte_off`` (16-byte aligned) on."""
        root = buf.root
        off = buf.base_off + byte_off
        es = DTYPE_BYTES[root.dtype]
        b = Buffer(root.kind, root.dtype, ((root.nbytes - off) // es,), name, base=root, base_off=off)
        self.buffers.append(b)
        return b

    def emit(self, kernel, operands, params, label, flops=0, nbytes=0) -> Record:
        r = Record(kernel, operands, params, label, flops, nbytes)
        idx = len(self.records)
        for b in operands:
            if b is not None:
                for x in (b, b.root):
                    if x.first < 0:
                        x.first = idx
                    x.last = idx
        self.records.append(r)
        return r

    def contiguous(self, value: Value) -> View:
        """Row-major view of ``value`` starting at its slot's first byte; a
        strided view is first copied to a new buffer, a row-major slice of a
        larger buffer gets a sub-range slot when 16-byte aligned."""
        v = self.views[value.name]
        if v.contiguous:
            return v
        if View(v.buf, v.shape, v.strides).contiguous:
            b = self.based(v, value.name)
            if b is not None:
                return b
        return self.copy_view(v, value.name + "_c")

    def based(self, v: View, name: str) -> Optional[View]:
        """``v`` with its element offset folded into a sub-range slot (offset 0),
        or None when the offset is not a multiple of 16 bytes."""
        if v.offset == 0:
            return v
        nbytes = v.offset * DTYPE_BYTES[v.buf.dtype]
        if (v.buf.base_off + nbytes) % 16:
            return None
        return View(self.alias(v.buf, nbytes, name + "@%d" % v.offset), v.shape, v.strides, 0)

    def padded_rows(self, value: Value, K: int) -> View:
        """[rows, K] copy of ``value`` (leading dims flattened) with rows Kp = ⌈K/8⌉·8 apart."""
        t = value.type
        rows = _prod(t.shape[:-1])
        Kp = (K + 7) // 8 * 8
        src = self.views[value.name]
        flat = view_reshape(src.shape, src.strides, (rows, K))
        if flat is not None and flat[1] == 1 and flat[0] % 8 == 0 and src.offset == 0:
            return View(src.buf, (rows, K), flat)  # rows already 16-byte strided
        if (src.buf.kind == "const" and src.buf.base is None and src.buf.name in self.const_tensors
                and flat is not None):
            import torch
            name = src.buf.name + "|pad%d" % Kp
            if name not in self.const_tensors:
                w = self.const_tensors[src.buf.name].reshape(-1).as_strided((rows, K), flat, src.offset)
                self.const_tensors[name] = torch.nn.functional.pad(w, (0, Kp - K))
            buf = self.derived_const(name, t.dtype, (rows, Kp))
            return View(buf, (rows, K), (Kp, 1))
        if flat is None:
            src = self.contiguous(value)
            flat = contiguous_strides((rows, K))
        out = View(self.new_buffer("arena", t.dtype, (rows, Kp), value.name + "_pad"), (rows, K), (Kp, 1))
        rb = RegionBuilder((rows, K))
        rb.store(out, rb.load(View(src.buf, (rows, K), flat, src.offset)))
        self.emit_region(rb, f"pad {value.name} K{K}->{Kp}")
        return out

    def copy_view_padded(self, v: View, new_shape: Tuple[int, ...], name: str) -> Optional[View]:
        """Materialise the reshape of ``v`` to ``new_shape`` (whose last dim K
        is a product of trailing dims of ``v``) with rows ⌈K/8⌉·8 elements
        apart, in one copy: the tensor-core operand layout of a linear input
        whose K is not a multiple of 8 (a conv patchify).  The pad columns are
        never read (the GEMM's operand map ends at K)."""
        K = new_shape[-1]
        acc, j = 1, len(v.shape)
        while j > 0 and acc < K:
            j -= 1
            acc *= v.shape[j]
        if acc != K:
            return None
        Kp = (K + 7) // 8 * 8
        rows = _prod(v.shape[:j])
        buf = self.new_buffer("arena", v.buf.dtype, (rows, Kp), name)
        dst = [0] * len(v.shape)
        step = 1
        for i in reversed(range(j, len(v.shape))):
            dst[i] = step
            step *= v.shape[i]
        step = Kp
        for i in reversed(range(j)):
            dst[i] = step
            step *= v.shape[i]
        rb = RegionBuilder(v.shape)
        rb.store(View(buf, v.shape, tuple(dst)), rb.load(v))
        self.emit_region(rb, f"copy {name} K{K}->{Kp}")
        nst = [1] * len(new_shape)
        step = Kp
        for i in reversed(range(len(new_shape) - 1)):
            nst[i] = step
            step *= new_shape[i]
        return View(buf, tuple(new_shape), tuple(nst))

    def copy_view(self, v: View, name: str) -> View:
        out = View(self.new_buffer("arena", v.buf.dtype, v.shape, name), v.shape, contiguous_strides(v.shape))
        rb = RegionBuilder(out.shape)
        r = rb.load(v)
        rb.store(out, r)
        self.emit_region(rb, f"copy {name}")
        return out

    def emit_region(self, rb: "RegionBuilder", label: str) -> None:
        desc, operands = rb.finish()
        nbytes = sum(b.nbytes for b in set(operands))
        self.emit(N.DP_K_REGION, operands, desc, label, 0, nbytes)

    # ------------------------------------------------------------- driver
    def run(self) -> Lowered:
        ins, consts = [], []
        for v in self.fn.inputs:
            if not isinstance(v.type, TensorType):
                raise CompilationError(f"input {v.name}: {v.type!r} is a host value; the GPU backend runs "
                                       "tensor programs only")
            kind = "const" if v.name in self.const_names else "input"
            b = self.new_buffer(kind, v.type.dtype, v.type.shape, v.name)
            self.views[v.name] = View(b, v.type.shape, contiguous_strides(v.type.shape))
            (consts if kind == "const" else ins).append((v.name, b))
        for op in self.fn.block.ops:
            if id(op) in self.done:
                continue
            self.lower_op(op)
            self.done.add(id(op))
        outs = self.bind_outputs()
        # constants no record reads (weights folded into a fused one) are not bound at all
        self.buffers = [b for b in self.buffers if not (b.kind == "const" and b.first < 0 and b.base is None)]
        consts = [(n, b) for n, b in consts if b.first >= 0] + \
                 [(n, b) for n, b in self.new_consts if b.first >= 0]
        arena = plan_arena(self.buffers)
        for i, b in enumerate(self.buffers):
            b.slot = i
        low = Lowered(self.fn.name, self.buffers, self.records, ins, consts, outs, arena)
        low.labels = [r.label for r in self.records]
        low.extra_consts = {n: self.const_tensors[n] for n, b in self.new_consts if b.first >= 0}
        return low

    def bind_outputs(self):
        outs, taken = [], set()
        if not self.fn.outputs:
            raise CompilationError("function has no output")
        for v in self.fn.outputs:
            view = self.views.get(v.name)
            if view is None:
                raise CompilationError(f"output {v.name} was never produced")
            shape = materialized_shape(v)
            if view.buf.kind == "arena" and view.contiguous and id(view.buf) not in taken \
                    and _prod(view.shape) == _prod(view.buf.shape):
                view.buf.kind = "output"
                view.buf.shape = tuple(shape)
                view.buf.name = v.name
                buf = view.buf
            else:
                buf = self.new_buffer("output", view.buf.dtype, shape, v.name)
                dst = View(buf, view.shape, contiguous_strides(view.shape))
                rb = RegionBuilder(view.shape)
                rb.store(dst, rb.load(view))
                self.emit_region(rb, f"output copy {v.name}")
            taken.add(id(buf))
            outs.append((v.name, buf))
        return outs

    def lower_op(self, op: Op) -> None:
        name = op.name
        if name in HOST_OPS:
            raise CompilationError(f"op '{name}' is a host string/tokenizer/dict op; the GPU backend does not "
                                   "execute it")
        if name == "resize":
            return self.lower_preproc(op)
        if name in ("linear", "matmul"):
            return self.lower_gemm(op)
        if name in ROW_OPS:
            return self.lower_rowreduce(op)
        if name == "embedding":
            return self.lower_embedding(op)
        if name == "reshape":
            out = op.outputs[0]
            shape = out.type.shape
            v = self.views[op.inputs[0].name]
            st = view_reshape(v.shape, v.strides, shape)
            if st is None:
                user = self.single_use(out)
                if (user is not None and user.name == "linear" and user.inputs[0] is out
                        and out.type.dtype == "bfloat16" and shape[-1] % 8):
                    pv = self.copy_view_padded(v, tuple(shape), out.name + "_pad")
                    if pv is not None:
                        self.views[out.name] = pv
                        return
                v = self.contiguous(op.inputs[0])
                st = contiguous_strides(shape)
            self.views[out.name] = View(v.buf, shape, st, v.offset)
            return
        if name == "transpose":
            v = self.views[op.inputs[0].name]
            dims = op.attr("dims")
            self.views[op.outputs[0].name] = View(v.buf, tuple(v.shape[d] for d in dims),
                                                  tuple(v.strides[d] for d in dims), v.offset)
            return
        if name == "slice":
            v = self.views[op.inputs[0].name]
            d, st = op.attr("dim"), op.attr("step")
            strides = list(v.strides)
            strides[d] *= st
            self.views[op.outputs[0].name] = View(v.buf, tuple(op.outputs[0].type.shape), tuple(strides),
                                                  v.offset + op.attr("start") * v.strides[d])
            return
        if name == "expand":
            v = self.views[op.inputs[0].name]
            shape = tuple(op.attr("shape"))
            lead = len(shape) - len(v.shape)
            strides = tuple(0 if i < lead or v.shape[i - lead] != s else v.strides[i - lead]
                            for i, s in enumerate(shape))
            self.views[op.outputs[0].name] = View(v.buf, shape, strides, v.offset)
            return
        if name == "cat":
            return self.lower_cat(op)
        if name == "rope":
            return self.lower_rope(op)
        if name in ELEMENTWISE:
            return self.lower_region(op)
        if name == "sdpa":
            return self.lower_sdpa(op)
        raise UnsupportedOpError(name)

    # --------------------------------------------------------- preprocess
    def lower_preproc(self, op: Op) -> None:
        x = self.contiguous(op.inputs[0])
        layout = op.attr("layout")
        if "C" not in layout:
            raise CompilationError(f"resize: layout {layout} has no channel dim")
        t_in = op.inputs[0].type
        in_shape = t_in.shape
        H, W = in_shape[layout.index("H")], in_shape[layout.index("W")]
        C = in_shape[layout.index("C")]
        B = in_shape[0] if layout.startswith("N") else 1
        oh, ow = op.attr("size")
        if C > 4:
            raise CompilationError("resize: at most 4 channels")
        if t_in.dtype not in ("uint8", "float32", "bfloat16", "float16"):
            raise CompilationError(f"resize: input dtype {t_in.dtype} unsupported")
        channels_last = layout in ("HWC", "NHWC")
        out_channels_last = channels_last
        out_dtype = op.outputs[0].type.dtype
        mean, std = None, None
        cur = op.outputs[0]
        chain_end = cur
        while True:
            nxt = self.single_use(cur)
            if nxt is None or id(nxt) in self.done:
                break
            if nxt.name == "to" and nxt.attr("dtype") in ("float32", "bfloat16", "float16"):
                if nxt.attr("dtype") != "float32" and mean is None and self._later_normalize(nxt):
                    break  # narrowing before a normalise would round early
                out_dtype = nxt.attr("dtype")
            elif nxt.name == "normalize" and mean is None and out_dtype == "float32":
                cd = nxt.attr("channel_dim")
                if nxt.attr("mean") is not None:
                    rank = len(nxt.inputs[0].type.shape)
                    want = (rank - 1) if out_channels_last else (rank - 3)
                    if cd != want:
                        break
                    mean, std = nxt.attr("mean"), nxt.attr("std")
                out_dtype = "float32"
            elif nxt.name == "transpose":
                dims = tuple(nxt.attr("dims"))
                rank = len(dims)
                to_planar = {3: (2, 0, 1), 4: (0, 3, 1, 2)}.get(rank)
                to_last = {3: (1, 2, 0), 4: (0, 2, 3, 1)}.get(rank)
                if out_channels_last and dims == to_planar:
                    out_channels_last = False
                elif not out_channels_last and dims == to_last:
                    out_channels_last = True
                else:
                    break
            else:
                break
            self.done.add(id(nxt))
            cur = nxt.outputs[0]
            chain_end = cur
        p = N.PreprocParams()
        p.batch, p.in_h, p.in_w, p.channels, p.out_h, p.out_w = B, H, W, C, oh, ow
        p.in_dtype = N.DTYPE_CODE[t_in.dtype]
        p.in_layout = N.DP_LAYOUT_NHWC if channels_last else N.DP_LAYOUT_NCHW
        p.out_dtype = N.DTYPE_CODE[out_dtype]
        p.out_layout = N.DP_LAYOUT_NHWC if out_channels_last else N.DP_LAYOUT_NCHW
        p.normalize = 1 if mean is not None else 0
        for c in range(4):
            p.mean[c] = mean[c] if mean is not None and c < C else 0.0
            p.stdv[c] = std[c] if std is not None and c < C else 1.0
        out = self.new_value_view(chain_end, dtype=out_dtype)
        in_bytes = B * C * H * W * DTYPE_BYTES[t_in.dtype]
        out_bytes = out.buf.nbytes
        self.emit(N.DP_K_PREPROC, [x.buf, out.buf], p,
                  f"preproc {layout}{'+norm' if mean is not None else ''} {H}x{W}->{oh}x{ow} {out_dtype}",
                  0, in_bytes + out_bytes)

    def _later_normalize(self, op: Op) -> bool:
        cur = op.outputs[0]
        for _ in range(4):
            nxt = self.single_use(cur)
            if nxt is None:
                return False
            if nxt.name == "normalize":
                return True
            cur = nxt.outputs[0]
        return False

    # --------------------------------------------------------------- GEMM
    def sibling_linears(self, op: Op) -> List[Op]:
        """Linears that read the same input as ``op`` with constant weights of
        the same K and dtype (the q/k/v projections of an attention block),
        in program order; ``[op]`` alone when there is nothing to fuse.  A
        linear whose output feeds an epilogue the GEMM would absorb (an
        activation, an add, a cast) is left on its own."""
        x = op.inputs[0]
        w0 = op.inputs[1]
        if not self.const_tensors or len(w0.type.shape) != 2:
            return [op]
        K = w0.type.shape[1]
        es = DTYPE_BYTES[op.outputs[0].type.dtype]

        def ok(u: Op) -> bool:
            if u.name != "linear" or id(u) in self.done or u.inputs[0].name != x.name:
                return False
            w = u.inputs[1]
            if (w.name not in self.const_tensors or len(w.type.shape) != 2 or w.type.shape[1] != K
                    or w.type.dtype != w0.type.dtype or (w.type.shape[0] * es) % 16):
                return False
            if (len(u.inputs) > 2) != (len(op.inputs) > 2):
                return False
            if len(u.inputs) > 2 and (u.inputs[2].name not in self.const_tensors
                                      or u.inputs[2].type.dtype != op.inputs[2].type.dtype):
                return False
            out = u.outputs[0]
            if out.type.dtype != op.outputs[0].type.dtype or out.name in self.out_names:
                return False
            return not any(c.name in ("relu", "gelu", "silu", "add", "to") for c in self.uses.get(out.name, []))

        group, seen = [], set()
        for u in self.uses.get(x.name, []):
            if id(u) not in seen and ok(u):
                seen.add(id(u))
                group.append(u)
        if op not in group or len(group) < 2:
            return [op]
        if w0.type.dtype == "bfloat16" and K % 8:
            return [op]
        return group

    def lower_linear_group(self, group: List[Op]) -> None:
        """One GEMM for sibling linears: their weights (and biases) are
        concatenated into one constant, and each output is a column block of
        the fused output, read in place through a sub-range slot."""
        import torch
        x_val = group[0].inputs[0]
        x = self.contiguous(x_val)
        K = group[0].inputs[1].type.shape[1]
        Ns = [u.inputs[1].type.shape[0] for u in group]
        Ntot = sum(Ns)

        def fused_const(idx: int, shape) -> View:
            name = "+".join(u.inputs[idx].name for u in group)
            if name not in self.const_tensors:
                self.const_tensors[name] = torch.cat([self.const_tensors[u.inputs[idx].name].reshape(-1, *shape[1:])
                                                      for u in group], 0)
            buf = self.derived_const(name, group[0].inputs[idx].type.dtype, shape)
            return View(buf, tuple(shape), contiguous_strides(tuple(shape)))

        w = fused_const(1, (Ntot, K))
        bias = fused_const(2, (Ntot,)) if len(group[0].inputs) > 2 else None
        lead = x.shape[:-1]
        out_dt = group[0].outputs[0].type.dtype
        out_shape = tuple(lead) + (Ntot,)
        out_buf = self.new_buffer("arena", out_dt, out_shape, "+".join(u.outputs[0].name for u in group))
        p = N.GemmParams()
        p.M, p.N, p.K = _prod(lead), Ntot, K
        p.lda = x.strides[-2] if len(x.shape) > 1 else K
        p.ldb, p.ldc = K, Ntot
        p.b_layout = N.DP_B_NK
        p.batch = 1
        a_dt = x.buf.dtype
        if a_dt != w.buf.dtype or a_dt not in ("float32", "bfloat16"):
            raise CompilationError(f"linear: operand dtypes {a_dt} x {w.buf.dtype}; supported: "
                                   "float32 x float32, bfloat16 x bfloat16")
        p.a_dtype = p.b_dtype = N.DTYPE_CODE[a_dt]
        p.c_dtype = N.DTYPE_CODE[out_dt]
        if bias is not None:
            p.epilogue = N.DP_EPI_BIAS
            p.bias_dtype = N.DTYPE_CODE[bias.buf.dtype]
        ops_ = [x.buf, w.buf, out_buf, bias.buf if bias is not None else None, None]
        self.emit(N.DP_K_GEMM, ops_, p, f"gemm linear x{len(group)} M{p.M} N{Ntot} K{K} {a_dt} epi{p.epilogue}",
                  2 * p.M * Ntot * K, sum(b.nbytes for b in ops_ if b is not None))
        es = DTYPE_BYTES[out_dt]
        strides = contiguous_strides(out_shape)
        col = 0
        for u, n in zip(group, Ns):
            v = u.outputs[0]
            buf = out_buf if col == 0 else self.alias(out_buf, col * es, v.name)
            self.views[v.name] = View(buf, tuple(lead) + (n,), strides)
            col += n
            self.done.add(id(u))

    # fp32 linears on the tensor cores: x·w = x_hi·w_hi + x_hi·w_lo + x_lo·w_hi
    # with *_hi the TF32-grid part (10 mantissa bits) and *_lo = * − *_hi,
    # run as ONE TF32 GEMM over K' = 3K on [x_hi | x_hi | x_lo] · [w_hi | w_lo | w_hi]ᵀ.
    # The dropped x_lo·w_lo term and the TF32 rounding of the lo parts are
    # ~2^-20 relative: fp32-level results (3xTF32).
    TF32_MIN_WORK = 1 << 24

    def tf32_split_ok(self, op: Op) -> bool:
        x, w = op.inputs[0], op.inputs[1]
        if x.type.dtype != "float32" or w.type.dtype != "float32" or len(w.type.shape) != 2:
            return False
        K = x.type.shape[-1]
        M = _prod(x.type.shape[:-1])
        src = self.views[w.name]
        const = (src.buf.kind == "const" and src.buf.base is None and src.buf.name in self.const_tensors)
        return const and K % 4 == 0 and M >= 64 and M * w.type.shape[0] * K >= self.TF32_MIN_WORK

    def tf32_split_weight(self, value: Value, K: int) -> View:
        import torch
        src = self.views[value.name]
        name = src.buf.name + "|3xtf32"
        if name not in self.const_tensors:
            rows = value.type.shape[0]
            flat = view_reshape(src.shape, src.strides, (rows, K)) or contiguous_strides((rows, K))
            w = self.const_tensors[src.buf.name].reshape(-1).as_strided((rows, K), flat, src.offset).float()
            hi = (w.contiguous().view(torch.int32) & -8192).view(torch.float32)
            self.const_tensors[name] = torch.cat([hi, w - hi, hi], dim=1).contiguous()
        buf = self.derived_const(name, "float32", (value.type.shape[0], 3 * K))
        return View(buf, (value.type.shape[0], 3 * K), (3 * K, 1))

    def tf32_fold_width(self, value: Value) -> int:
        """K when ``value``'s only consumer is a linear that runs as 3xTF32 with
        ``value`` as its activation (possibly through single-use reshapes that
        keep the last dim), so that the producer can write the [hi | hi | lo]
        operand itself instead of ``value`` (0 otherwise)."""
        K = value.type.shape[-1]
        v, nxt = value, self.single_use(value)
        while (nxt is not None and nxt.name == "reshape" and id(nxt) not in self.done
               and nxt.outputs[0].type.shape[-1] == K):
            v = nxt.outputs[0]
            nxt = self.single_use(v)
        if (nxt is None or nxt.name != "linear" or nxt.inputs[0].name != v.name
                or value.type.dtype != "float32" or len(self.sibling_linears(nxt)) > 1
                or not self.tf32_split_ok(nxt)):
            return 0
        return K

    def new_tf32_split_view(self, value: Value, K: int) -> View:
        """The [rows, 3K] operand buffer that ``value``'s producer writes; the
        reshapes between ``value`` and its linear are consumed here."""
        rows = _prod(value.type.shape[:-1])
        out = self.new_buffer("arena", "float32", (rows, 3 * K), value.name + "_3xtf32")
        view = View(out, (rows, 3 * K), (3 * K, 1))
        v = value
        self.tf32_split_views[v.name] = view
        nxt = self.single_use(v)
        while nxt is not None and nxt.name == "reshape":
            self.done.add(id(nxt))
            v = nxt.outputs[0]
            self.tf32_split_views[v.name] = view
            nxt = self.single_use(v)
        return view

    def tf32_split_rows(self, value: Value, K: int) -> View:
        """[rows, 3K] = [x_hi | x_hi | x_lo]: written by the producer when it
        could (embedding, split-K reduce, row norm), else one region."""
        if value.name in self.tf32_split_views:
            return self.tf32_split_views[value.name]
        rows = _prod(value.type.shape[:-1])
        src = self.views[value.name]
        flat = view_reshape(src.shape, src.strides, (rows, K))
        if flat is None:
            src = self.contiguous(value)
            flat = contiguous_strides((rows, K))
        out = self.new_buffer("arena", "float32", (rows, 3 * K), value.name + "_3xtf32")
        rb = RegionBuilder((rows, K))
        xr = rb.load(View(src.buf, (rows, K), flat, src.offset))
        hi = rb.unary("tf32", xr)
        rb.store(View(out, (rows, K), (3 * K, 1), 0), hi)
        rb.store(View(out, (rows, K), (3 * K, 1), K), hi)
        rb.store(View(out, (rows, K), (3 * K, 1), 2 * K), rb.binary("sub", xr, hi))
        self.emit_region(rb, f"split {value.name} 3xtf32")
        return View(out, (rows, 3 * K), (3 * K, 1))

    def lower_gemm(self, op: Op) -> None:
        p = N.GemmParams()
        tf32 = False
        if op.name == "linear":
            group = self.sibling_linears(op)
            if len(group) > 1:
                return self.lower_linear_group(group)
            K = op.inputs[0].type.shape[-1]
            tf32 = self.tf32_split_ok(op)
            if tf32:
                x = self.tf32_split_rows(op.inputs[0], K)
                w = self.tf32_split_weight(op.inputs[1], K)
            elif op.inputs[0].type.dtype == "bfloat16" and K % 8:
                # tensor-core operands need 16-byte row strides: rows padded to Kp
                x = self.padded_rows(op.inputs[0], K)
                w = self.padded_rows(op.inputs[1], K)
            else:
                x = self.contiguous(op.inputs[0])
                w = self.contiguous(op.inputs[1])
            M = _prod(x.shape[:-1])
            Nn = w.shape[0]
            p.M, p.N, p.K = M, Nn, x.shape[-1]
            p.lda, p.ldb = x.strides[-2] if len(x.shape) > 1 else x.shape[-1], w.strides[0]
            p.b_layout = N.DP_B_NK
            p.batch, p.stride_a, p.stride_b = 1, 0, 0
            a_dtype, b_dtype = x.buf.dtype, w.buf.dtype
            a_buf, b_buf = x, w
            bias = None
            if len(op.inputs) > 2:
                bias = self.contiguous(op.inputs[2])
        else:
            a = self.contiguous(op.inputs[0])
            bview = self.views[op.inputs[1].name]
            ta, tb = op.inputs[0].type, op.inputs[1].type
            M, K = ta.shape[-2], ta.shape[-1]
            Nn = tb.shape[-1]
            batch_a, batch_b = ta.shape[:-2], tb.shape[:-2]
            # B as [N, K] when it is a transposed view of a row-major [N, K] tensor.
            bs = bview.strides
            if bs[-2] == 1 and bs[-1] == K and bview.offset == 0 and _prod(batch_b) == 1:
                b_buf, p.b_layout, p.ldb = bview, N.DP_B_NK, K
            else:
                b_buf = self.contiguous(op.inputs[1])
                p.b_layout, p.ldb = N.DP_B_KN, Nn
            bb = _prod(batch_b)
            ba = _prod(batch_a)
            if bb == 1:
                # fold A's batch dims into M
                M = M * ba
                p.batch, p.stride_a, p.stride_b = 1, 0, 0
            elif ba == bb and batch_a == batch_b:
                p.batch, p.stride_a, p.stride_b = ba, M * K, K * Nn
            else:
                raise CompilationError(f"matmul: batch broadcast {batch_a} x {batch_b} unsupported")
            p.M, p.N, p.K = M, Nn, K
            p.lda = K
            a_dtype, b_dtype = a.buf.dtype, b_buf.buf.dtype
            a_buf = a
            bias = None
        if a_dtype != b_dtype or a_dtype not in ("float32", "bfloat16"):
            raise CompilationError(f"{op.name}: operand dtypes {a_dtype} x {b_dtype}; supported: "
                                   "float32 x float32, bfloat16 x bfloat16")
        p.a_dtype = p.b_dtype = N.DP_TF32 if tf32 else N.DTYPE_CODE[a_dtype]
        epi = 0
        residual = None
        shared_rows = 0
        c_dtype = op.outputs[0].type.dtype
        if bias is not None:
            epi |= N.DP_EPI_BIAS
        act_done = False
        cur = op.outputs[0]
        out_shape = tuple(op.outputs[0].type.shape)
        # The GEMM output as seen through the reshape / transpose views between it
        # and the next elementwise op; that op fuses only while this stays the
        # plain row-major layout of the GEMM's own output.
        sym = (out_shape, contiguous_strides(out_shape))
        pending: List[Op] = []
        argmax_op = None
        while True:
            nxt = self.single_use(cur)
            if nxt is None or id(nxt) in self.done:
                break
            if nxt.name in ("reshape", "transpose"):
                shp, st = sym
                if nxt.name == "reshape":
                    new_shape = tuple(nxt.outputs[0].type.shape)
                    nst = view_reshape(shp, st, new_shape)
                    if nst is None:
                        break
                    sym = (new_shape, tuple(nst))
                else:
                    dims = nxt.attr("dims")
                    sym = (tuple(shp[d] for d in dims), tuple(st[d] for d in dims))
                pending.append(nxt)
                cur = nxt.outputs[0]
                continue
            shp, st = sym
            if not View(None, shp, st).contiguous:
                break
            last = False
            if nxt.name == "add":
                other = nxt.inputs[1] if nxt.inputs[0] is cur else nxt.inputs[0]
                if other is cur:
                    break
                ot = other.type
                if tuple(nxt.outputs[0].type.shape) != shp:
                    break
                if (bias is None and not act_done and residual is None and ot.shape[-1:] == (p.N,)
                        and shp[-1] == p.N and _prod(ot.shape) == p.N):
                    bias = self.contiguous(other)
                    epi |= N.DP_EPI_BIAS
                elif residual is None and tuple(ot.shape) == shp and ot.dtype in FLOAT_DTYPES:
                    residual = self.contiguous(other)
                    epi |= N.DP_EPI_RESIDUAL
                elif (residual is None and ot.dtype in FLOAT_DTYPES and op.name == "linear" and p.batch == 1
                      and len(shp) >= 3 and shp[-1] == p.N and tuple(ot.shape[-2:]) == shp[-2:]
                      and _prod(ot.shape[:-2]) == 1):
                    # a [1, T, N] addend shared by every sample (a position embedding):
                    # the GEMM runs as M/T batches of T rows with a batch-shared residual
                    residual = self.contiguous(other)
                    epi |= N.DP_EPI_RESIDUAL
                    shared_rows = shp[-2]
                else:
                    break
                c_dtype = nxt.outputs[0].type.dtype
            elif nxt.name == "mul" and residual is None and not shared_rows:
                # a gated unit: this GEMM times an already computed same-shape operand
                # (gelu(gate) · up of a GeGLU MLP, with the gate GEMM lowered first)
                other = nxt.inputs[1] if nxt.inputs[0] is cur else nxt.inputs[0]
                if (other is cur or tuple(other.type.shape) != shp or other.type.dtype not in FLOAT_DTYPES
                        or tuple(nxt.outputs[0].type.shape) != shp or not self.ready(other)):
                    break
                residual = self.contiguous(other)
                epi |= N.DP_EPI_MUL
                c_dtype = nxt.outputs[0].type.dtype
            elif nxt.name in ("relu", "gelu", "silu") and not act_done and residual is None:
                if nxt.name == "relu":
                    epi |= N.DP_EPI_RELU
                elif nxt.name == "silu":
                    epi |= N.DP_EPI_SILU
                else:
                    epi |= N.DP_EPI_GELU_TANH if nxt.attr("approximate") == "tanh" else N.DP_EPI_GELU_ERF
                act_done = True
            elif nxt.name == "to" and nxt.attr("dtype") in ("float32", "bfloat16", "float16"):
                c_dtype = nxt.attr("dtype")
                last = True
            elif (nxt.name == "argmax" and op.name == "linear" and p.batch == 1 and not shared_rows
                  and (tf32 or a_dtype == "bfloat16") and len(shp) >= 1 and shp[-1] == p.N
                  and nxt.attr("dim", -1) % len(shp) == len(shp) - 1 and not nxt.attr("keepdim", False)):
                # the row argmax of the GEMM's result, reduced in the epilogue: the logits are never stored
                argmax_op = nxt
                last = True
            else:
                break
            for v in pending:
                self.done.add(id(v))
            pending = []
            self.done.add(id(nxt))
            cur = nxt.outputs[0]
            if argmax_op is not None:
                break
            out_shape = tuple(cur.type.shape)
            sym = (out_shape, contiguous_strides(out_shape))
            if last:
                break
        if pending:  # views after the last fused op stay ordinary views of its output
            cur = pending[0].inputs[0]
        p.epilogue = epi
        p.c_dtype = N.DTYPE_CODE[c_dtype]
        if shared_rows:
            p.batch, p.M = p.M // shared_rows, shared_rows
            p.stride_a, p.stride_b = shared_rows * p.lda, 0
        p.ldc = p.N
        p.stride_c = p.M * p.N if p.batch > 1 else 0
        if bias is not None:
            p.bias_dtype = N.DTYPE_CODE[bias.buf.dtype]
        if residual is not None:
            p.r_dtype = N.DTYPE_CODE[residual.buf.dtype]
            p.ldr = p.N
            p.stride_r = p.M * p.N if p.batch > 1 and not shared_rows else 0
        if argmax_op is not None:
            return self.emit_gemm_argmax(op, p, tf32, a_dtype, a_buf, b_buf, bias, residual, c_dtype, cur)
        out = self.new_value_view(cur, dtype=c_dtype)
        flops = 2 * p.M * p.N * p.K * p.batch
        ops_ = [a_buf.buf, b_buf.buf, out.buf, bias.buf if bias is not None else None,
                residual.buf if residual is not None else None]
        nb = sum(b.nbytes for b in ops_ if b is not None)
        kind = "3xtf32" if tf32 else a_dtype
        if tf32:
            flops = 2 * p.M * p.N * (p.K // 3) * p.batch  # the work of the fp32 product
        label = f"gemm {op.name} M{p.M} N{p.N} K{p.K} b{p.batch} {kind} epi{epi}"
        splits = 1
        if p.batch == 1 and not shared_rows and not (epi & N.DP_EPI_SOFTMAX) and (tf32 or a_dtype == "bfloat16"):
            splits = splitk_factor(p.M, p.N, p.K, tf32, p.b_layout)
        if splits == 1:
            skb = streamk_bytes(p.M, p.N, p.K, p.batch, tf32, epi) if (tf32 or a_dtype == "bfloat16") else 0
            if skb and self.use_streamk:
                # Tiles past the last full wave split by K stage over every CTA group.
                sp = N.StreamKParams()
                sp.gemm, sp.workspace_bytes = p, skb
                ws = self.new_buffer("arena", "uint8", (skb,), f"{cur.name}_streamk")
                self.emit(N.DP_K_GEMM_SK, ops_ + [ws], sp, f"{label} streamk", flops, nb)
            else:
                self.emit(N.DP_K_GEMM, ops_, p, label, flops, nb)
            return
        # Split K: a batched GEMM over the K slices writes raw fp32 partial
        # products to a workspace [S, M, N]; the reduce record sums them in
        # slice order and applies the epilogue.
        ws = self.new_buffer("arena", "float32", (splits, p.M, p.N), f"{cur.name}_splitk")
        g = N.GemmParams.from_buffer_copy(bytes(p))
        ks = p.K // splits
        g.K, g.batch = ks, splits
        g.stride_a = ks
        g.stride_b = ks if p.b_layout == N.DP_B_NK else ks * p.ldb
        g.c_dtype, g.ldc, g.stride_c = N.DP_F32, p.N, p.M * p.N
        g.epilogue, g.alpha, g.bias_dtype, g.r_dtype, g.ldr, g.stride_r = 0, 0.0, 0, 0, 0, 0
        self.emit(N.DP_K_GEMM, [a_buf.buf, b_buf.buf, ws, None, None], g, f"{label} splitk{splits}", flops,
                  nb - out.buf.nbytes + ws.nbytes)
        sp = N.SplitKParams()
        sp.gemm = p
        sp.splits, sp.slice_stride = splits, p.M * p.N
        split_note = ""
        K = self.tf32_fold_width(cur) if c_dtype == "float32" and not (epi & N.DP_EPI_ARGMAX) else 0
        if K == p.N and cur.name in self.views and self.views[cur.name] is out and out.buf.first < 0:
            # Feeding a 3xTF32 linear: the reduce stores [hi | hi | lo] rows.
            del self.views[cur.name]
            self.buffers.remove(out.buf)
            out = self.new_tf32_split_view(cur, K)
            sp.gemm.epilogue |= N.DP_EPI_TF32SPLIT
            sp.gemm.ldc = 3 * p.N
            split_note = " -> 3xtf32 operand"
        self.emit(N.DP_K_SPLITK, [ws, out.buf, bias.buf if bias is not None else None,
                                  residual.buf if residual is not None else None], sp,
                  f"splitk reduce {splits}x{p.M}x{p.N} epi{epi}{split_note}", 0, ws.nbytes + out.buf.nbytes)

    def emit_gemm_argmax(self, op, p, tf32, a_dtype, a_buf, b_buf, bias, residual, logits_dtype, idx_val) -> None:
        """A linear whose only consumer is a row argmax: three records - clear
        one uint64 key per row, the GEMM with the argmax epilogue (each tile
        folds its rows' (value, first column) into the keys by atomicMax), and
        the keys to indices (with a following int cast folded in)."""
        idx_dtype = idx_val.type.dtype
        nxt = self.single_use(idx_val)
        if nxt is not None and nxt.name == "to" and nxt.attr("dtype") in ("int32", "int64"):
            idx_dtype = nxt.attr("dtype")
            self.done.add(id(nxt))
            idx_val = nxt.outputs[0]
        keys = self.new_buffer("arena", "int64", (p.M,), f"{idx_val.name}_keys")
        self.emit(N.DP_K_ARGMAX_KEYS, [keys, None], N.ArgmaxKeysParams(p.M, 0, 0), f"argmax keys clear {p.M}", 0,
                  keys.nbytes)
        p.epilogue |= N.DP_EPI_ARGMAX
        p.c_dtype = N.DTYPE_CODE[logits_dtype]
        p.ldc, p.stride_c = p.N, 0
        if bias is not None:
            p.bias_dtype = N.DTYPE_CODE[bias.buf.dtype]
        if residual is not None:
            p.r_dtype = N.DTYPE_CODE[residual.buf.dtype]
            p.ldr = p.N
        ops_ = [a_buf.buf, b_buf.buf, keys, bias.buf if bias is not None else None,
                residual.buf if residual is not None else None]
        flops = 2 * p.M * p.N * (p.K // 3 if tf32 else p.K)
        kind = "3xtf32" if tf32 else a_dtype
        self.emit(N.DP_K_GEMM, ops_, p, f"gemm {op.name} M{p.M} N{p.N} K{p.K} b1 {kind} epi{p.epilogue} argmax",
                  flops, sum(b.nbytes for b in ops_ if b is not None))
        out = self.new_value_view(idx_val, dtype=idx_dtype)
        self.emit(N.DP_K_ARGMAX_KEYS, [keys, out.buf], N.ArgmaxKeysParams(p.M, 1, N.DTYPE_CODE[idx_dtype]),
                  f"argmax keys -> {idx_dtype} {p.M}", 0, keys.nbytes + out.buf.nbytes)

    # ------------------------------------------------------ row reductions
    def lower_rowreduce(self, op: Op) -> None:
        x_val = op.inputs[0]
        t = x_val.type
        rank = len(t.shape)
        dim = op.attr("dim", -1)
        if op.name in ("layer_norm", "rms_norm"):
            dim = -1
        d = dim % rank
        xv = self.views[x_val.name]
        cols = t.shape[d]
        rows = t.numel // cols
        row_stride = cols
        if d != rank - 1:
            # move the reduced dim last with a strided copy
            perm = [i for i in range(rank) if i != d] + [d]
            xv = self.copy_view(View(xv.buf, tuple(xv.shape[i] for i in perm),
                                     tuple(xv.strides[i] for i in perm), xv.offset), x_val.name + "_t")
        elif not xv.contiguous:
            # rows of unit-stride elements a fixed distance apart are read in place
            flat = view_reshape(xv.shape, xv.strides, (rows, cols))
            based = self.based(xv, x_val.name) if flat is not None and (flat[1] == 1 or cols == 1) else None
            if based is not None:
                xv, row_stride = based, flat[0]
            else:
                xv = self.copy_view(xv, x_val.name + "_c")
        if t.dtype not in ("float32", "bfloat16", "float16"):
            raise CompilationError(f"{op.name}: input dtype {t.dtype} unsupported (float types only)")
        p = N.RowReduceParams()
        p.rows, p.cols, p.in_row_stride = rows, cols, row_stride
        p.in_dtype = N.DTYPE_CODE[t.dtype]
        kind = {"sum": N.DP_RED_SUM, "max": N.DP_RED_MAX, "min": N.DP_RED_MIN, "mean": N.DP_RED_MEAN,
                "argmax": N.DP_RED_ARGMAX, "softmax": N.DP_RED_SOFTMAX, "rms_norm": N.DP_RED_RMSNORM,
                "layer_norm": N.DP_RED_LAYERNORM}[op.name]
        p.kind = kind
        w = b = None
        out_val = op.outputs[0]
        if op.name == "argmax":
            out_dtype = out_val.type.dtype
            nxt = self.single_use(out_val)
            if nxt is not None and nxt.name == "to" and nxt.attr("dtype") in ("int32", "int64"):
                out_dtype = nxt.attr("dtype")
                self.done.add(id(nxt))
                out_val = nxt.outputs[0]
            p.out_row_stride = 1
        elif op.name in ("sum", "max", "min", "mean"):
            out_dtype = out_val.type.dtype
            p.out_row_stride = 1
        else:
            out_dtype = out_val.type.dtype
            p.out_row_stride = cols
            if op.name == "layer_norm":
                p.eps = op.attr("eps")
                idx = 1
                if op.attr("has_weight"):
                    w = self._param_like(op.inputs[idx], t.dtype)
                    idx += 1
                if op.attr("has_bias"):
                    b = self._param_like(op.inputs[idx], t.dtype)
            elif op.name == "rms_norm":
                p.eps = op.attr("eps")
                p.weight_offset = op.attr("weight_offset", 0.0)
                if op.attr("has_weight"):
                    w = self._param_like(op.inputs[1], t.dtype)
            p.has_weight = 1 if w is not None else 0
            p.has_bias = 1 if b is not None else 0
        p.out_dtype = N.DTYPE_CODE[out_dtype]
        K = self.tf32_fold_width(out_val) if op.name in ("softmax", "layer_norm", "rms_norm") else 0
        if K and t.dtype == "float32" and out_dtype == "float32" and d == rank - 1 and cols <= 4096:
            # Feeding a 3xTF32 linear: rows stored as [hi | hi | lo].
            out = self.new_tf32_split_view(out_val, K)
            p.out_split, p.out_row_stride = 1, 3 * cols
        else:
            out = self.new_value_view(out_val, dtype=out_dtype)
        nbytes = xv.buf.nbytes + out.buf.nbytes
        self.emit(N.DP_K_ROWREDUCE, [xv.buf, w.buf if w else None, b.buf if b else None, out.buf], p,
                  f"rowreduce {op.name} {rows}x{cols} {t.dtype}->{out_dtype}{' 3xtf32 operand' if p.out_split else ''}",
                  0, nbytes)

    def _param_like(self, value: Value, dtype: str) -> View:
        v = self.contiguous(value)
        if v.buf.dtype == dtype:
            return v
        out = View(self.new_buffer("arena", dtype, v.shape, value.name + "_cast"), v.shape,
                   contiguous_strides(v.shape))
        rb = RegionBuilder(v.shape)
        rb.store(out, rb.load(v))
        self.emit_region(rb, f"cast {value.name} to {dtype}")
        return out

    # ------------------------------------------------------------ attention
    def lower_sdpa(self, op: Op) -> None:
        """softmax(Q·Kᵀ·scale)·V as two batched tensor-core GEMMs around a row softmax.

        Q [.., Hq, L, D], K [.., Hk, S, D], V [.., Hk, S, Dv], Hq a multiple of Hk
        (grouped-query attention: the Hq/Hk query heads of a group share one K/V
        head, so each group is one GEMM of (Hq/Hk)·L rows).  Scores are fp32,
        probabilities are stored in the operand dtype.
        """
        if op.attr("is_causal"):
            raise CompilationError("sdpa: causal masking is not supported yet")
        q, k, v = op.inputs
        tq, tk, tv = q.type, k.type, v.type
        if len(tq.shape) < 3:
            raise CompilationError("sdpa: inputs need [.., heads, len, dim]")
        Hq, L, D = tq.shape[-3:]
        Hk, S, Dk = tk.shape[-3:]
        Dv = tv.shape[-1]
        B = _prod(tq.shape[:-3])
        if Dk != D or tv.shape[-2] != S or tv.shape[-3] != Hk or Hq % Hk:
            raise CompilationError("sdpa: inconsistent q/k/v shapes")
        if tq.dtype != tk.dtype or tq.dtype != tv.dtype or tq.dtype not in ("bfloat16", "float32"):
            raise CompilationError("sdpa: q, k, v must share dtype bf16 or fp32")
        g = Hq // Hk
        dt = tq.dtype

        def operand(value: Value, rows_shape):
            """(view, strides as [B, H, rows, D]) of an operand read in place when
            its strides and start allow it (a slice of a fused projection)."""
            vw = self.views[value.name]
            st = view_reshape(vw.shape, vw.strides, rows_shape)
            based = None
            if st is not None and st[3] == 1 and not any(x % 8 for x in st[:3]):
                based = self.based(vw, value.name)
            if based is None:
                vw = self.contiguous(value)
                st = view_reshape(vw.shape, vw.strides, rows_shape) or contiguous_strides(rows_shape)
                return vw, st
            return based, st

        if g == 1:
            qv, qst = operand(q, (B, Hq, L, D))
            q_b, q_b2, q_ld = qst[0], qst[1], qst[2]
            rows_q, batch, batch2 = L, B * Hq, Hq
        else:
            # Query heads of one group stacked as one (g·L)-row operand: in place
            # when a group's g·L rows are evenly strided (head stride = L · row stride).
            qv, qst = operand(q, (B, Hq, L, D))
            if qst[1] != L * qst[2]:
                qv = self.contiguous(q)
                qst = contiguous_strides((B, Hq, L, D))
            q_b, q_b2, q_ld = qst[0], g * qst[1], qst[2]
            rows_q, batch, batch2 = g * L, B * Hk, Hk
        kv, kst = operand(k, (B, Hk, S, D))
        # V is read in place as the GEMM's [K = keys, N = Dv] operand (N contiguous)
        vv, vst = operand(v, (B, Hk, S, Dv))
        if self.use_fused_attention and dt == "bfloat16" and D <= 256 and Dv <= 256 and D % 8 == 0 \
                and Dv % 8 == 0:
            return self.lower_attention_fused(op, qv, (q_b, q_b2 // g if g > 1 else q_b2, q_ld), kv, kst, vv, vst,
                                              B, Hq, Hk, g, L, S, D, Dv)
        # bf16 rows of at most 256 keys: the score GEMM's epilogue computes the row
        # softmax itself (one tensor-core tile holds a whole row) and writes bf16
        # probabilities; otherwise fp32 scores go through a separate row softmax.
        fused = dt == "bfloat16" and S <= 256
        # Score / probability rows padded to Sp = ⌈S/8⌉·8 columns so the value
        # GEMM reads them as a tensor-core operand; the pad is never read
        # (the operand maps end at S).
        Sp = (S + 7) // 8 * 8
        probs = View(self.new_buffer("arena", dt, (batch, rows_q, Sp), op.outputs[0].name + "_p"),
                     (batch, rows_q, S), (rows_q * Sp, Sp, 1))
        if fused:
            scores = probs
        else:
            scores = View(self.new_buffer("arena", "float32", (batch, rows_q, Sp), op.outputs[0].name + "_s"),
                          (batch, rows_q, S), (rows_q * Sp, Sp, 1))
        p = N.GemmParams()
        p.M, p.N, p.K = rows_q, S, D
        p.lda, p.ldb, p.ldc = q_ld, kst[2], Sp
        p.batch, p.batch2 = batch, batch2
        p.stride_a, p.stride_a2 = q_b, q_b2
        p.stride_b, p.stride_b2 = kst[0], kst[1]
        p.stride_c, p.stride_c2 = batch2 * rows_q * Sp, rows_q * Sp
        p.a_dtype = p.b_dtype = N.DTYPE_CODE[dt]
        p.c_dtype = N.DTYPE_CODE[dt] if fused else N.DP_F32
        p.b_layout = N.DP_B_NK
        p.alpha = float(op.attr("scale"))
        p.epilogue = N.DP_EPI_SOFTMAX if fused else 0
        self.emit(N.DP_K_GEMM, [qv.buf, kv.buf, scores.buf, None, None], p,
                  f"gemm attn-scores{'+softmax' if fused else ''} b{batch} M{rows_q} N{S} K{D} {dt}",
                  2 * B * Hq * L * S * D, qv.buf.nbytes + kv.buf.nbytes + scores.buf.nbytes)
        if not fused:
            r = N.RowReduceParams()
            r.kind, r.in_dtype, r.out_dtype = N.DP_RED_SOFTMAX, N.DP_F32, N.DTYPE_CODE[dt]
            r.rows, r.cols, r.in_row_stride, r.out_row_stride = B * Hq * L, S, Sp, Sp
            self.emit(N.DP_K_ROWREDUCE, [scores.buf, None, None, probs.buf], r,
                      f"rowreduce attn-softmax {B * Hq * L}x{S}", 0, scores.buf.nbytes + probs.buf.nbytes)
        p2 = N.GemmParams()
        p2.M, p2.N, p2.K = rows_q, Dv, S
        p2.lda, p2.ldb = Sp, vst[2]
        p2.batch, p2.batch2 = batch, batch2
        p2.stride_a, p2.stride_a2 = batch2 * rows_q * Sp, rows_q * Sp
        p2.stride_b, p2.stride_b2 = vst[0], vst[1]
        p2.a_dtype = p2.b_dtype = p2.c_dtype = N.DTYPE_CODE[dt]
        p2.b_layout = N.DP_B_KN
        out_v = op.outputs[0]
        if g == 1 and len(tq.shape) == 4:
            # Store token-major [B, L, Hq, Dv]; the value is its [B, Hq, L, Dv] view, so the
            # usual transpose(1, 2).reshape(B, L, Hq·Dv) that follows costs nothing.
            buf = self.new_buffer("arena", dt, (B, L, Hq, Dv), out_v.name)
            self.views[out_v.name] = View(buf, (B, Hq, L, Dv), (L * Hq * Dv, Dv, Hq * Dv, 1))
            p2.ldc, p2.stride_c, p2.stride_c2 = Hq * Dv, L * Hq * Dv, Dv
        else:
            buf = self.new_value_view(out_v).buf
            p2.ldc, p2.stride_c, p2.stride_c2 = Dv, Hk * rows_q * Dv, rows_q * Dv
        self.emit(N.DP_K_GEMM, [probs.buf, vv.buf, buf, None, None], p2,
                  f"gemm attn-values b{batch} M{rows_q} N{Dv} K{S} {dt}", 2 * B * Hq * L * S * Dv,
                  probs.buf.nbytes + vv.buf.nbytes + buf.nbytes)

    # ---------------------------------------------------------- cat / rope
    def lower_cat(self, op: Op) -> None:
        """One copy region per input into its slice of the output buffer.

        A cat whose first input is the same value as an earlier cat's (a
        layer's prefix keys, concatenated with new keys at every denoise step)
        reuses that cat's buffer once nothing reads the earlier result any
        more, and copies only the inputs that differ: the shared prefix is
        written once."""
        d = op.attr("dim")
        out_val = op.outputs[0]
        key = (d, tuple(out_val.type.shape), out_val.type.dtype, op.inputs[0].name)
        prev = self.cat_reuse.get(key)
        same = [False] * len(op.inputs)
        out = None
        if prev is not None:
            prev_view, prev_name, prev_inputs = prev
            if (prev_name not in self.out_names and len(prev_inputs) == len(op.inputs)
                    and not self.buffer_read_later(prev_view.buf, op)):
                out = prev_view
                self.views[out_val.name] = out
                same = [a == v.name for a, v in zip(prev_inputs, op.inputs)]
        if out is None:
            out = self.new_value_view(out_val)
        if out.contiguous and out_val.name not in self.out_names:
            self.cat_reuse[key] = (out, out_val.name, [v.name for v in op.inputs])
        pos = 0
        for v, kept in zip(op.inputs, same):
            src = self.views[v.name]
            n = v.type.shape[d]
            if n and not kept:
                dst = View(out.buf, src.shape, out.strides, out.offset + pos * out.strides[d])
                rb = RegionBuilder(src.shape)
                rb.store(dst, rb.load(src))
                self.emit_region(rb, f"cat {v.name} -> {op.outputs[0].name}[{pos}:{pos + n}]")
            pos += n

    def buffer_read_later(self, buf: Buffer, current: Op) -> bool:
        """Whether an op not lowered yet (other than ``current``) reads a value
        whose view lies in ``buf`` (any view of it: reshapes, transposes and
        slices alias it), or a function output does."""
        def aliases(name: str) -> bool:
            v = self.views.get(name)
            return v is not None and (v.buf is buf or v.buf.root is buf)
        ops = self.fn.block.ops
        start = self.op_index.get(id(current), -1) + 1  # every op before the current one is lowered
        for o in ops[start:]:
            if id(o) in self.done:
                continue
            if any(aliases(v.name) for v in o.inputs):
                return True
        return any(aliases(n) for n in self.out_names)

    def lower_rope(self, op: Op) -> None:
        """out1 = x1·c1 − x2·s1, out2 = x2·c2 + x1·s2 over the two halves of the
        last dim, as one region over the half shape with six loads and two
        stores (c1 = c2, s1 = s2 for half-width tables)."""
        x_val, c_val, s_val = op.inputs
        xv = self.views[x_val.name]
        if self.lower_rope_kernel(op):
            return
        D = x_val.type.shape[-1]
        h = D // 2
        half = tuple(x_val.type.shape[:-1]) + (h,)

        def halves(v: View):
            lo = View(v.buf, tuple(v.shape[:-1]) + (h,) if v.shape[-1] == D else tuple(v.shape), v.strides,
                      v.offset)
            if v.shape[-1] == h:
                return lo, lo
            return lo, View(v.buf, lo.shape, v.strides, v.offset + h * v.strides[-1])

        x1, x2 = halves(xv)
        c1, c2 = halves(self.views[c_val.name])
        s1, s2 = halves(self.views[s_val.name])
        out = self.new_value_view(op.outputs[0])
        o1, o2 = halves(out)
        rb = RegionBuilder(half)
        rx1, rx2 = rb.load(x1), rb.load(x2)
        lo = rb.binary("sub", rb.binary("mul", rx1, rb.load(c1)), rb.binary("mul", rx2, rb.load(s1)))
        rb.store(o1, lo)
        rb.release(lo)
        hi = rb.binary("add", rb.binary("mul", rx2, rb.load(c2)), rb.binary("mul", rx1, rb.load(s2)))
        rb.store(o2, hi)
        self.emit_region(rb, f"rope {half}")

    def lower_rope_kernel(self, op: Op) -> bool:
        """One ``dp_rope`` record when x is at most 4-d with a contiguous last
        dim, the two tables share one broadcast layout, and every base, stride
        and half width is 16-byte vector aligned; False leaves the region."""
        x_val, c_val, s_val = op.inputs
        xv, cv, sv = (self.views[v.name] for v in op.inputs)
        dt, tdt = x_val.type.dtype, c_val.type.dtype
        if dt not in ("bfloat16", "float16", "float32") or tdt != s_val.type.dtype or \
                tdt not in ("bfloat16", "float16", "float32"):
            return False
        rank, D = len(xv.shape), xv.shape[-1]
        if rank > 4 or D % 2 or xv.strides[-1] != 1:
            return False
        vec = 16 // DTYPE_BYTES[dt]
        tb = DTYPE_BYTES[tdt]
        t_align = 16 // tb if vec * tb >= 16 else vec
        if (D // 2) % vec:
            return False

        def table(v: View):
            """(strides over x's 4 dims, half_table) of a table broadcast to x."""
            if v.shape[-1] not in (D, D // 2) or v.strides[-1] != 1:
                return None
            lead = rank - len(v.shape)
            if lead < 0:
                return None
            st = []
            for k in range(rank - 1):
                j = k - lead
                if j < 0 or v.shape[j] == 1:
                    st.append(0)
                elif v.shape[j] == xv.shape[k]:
                    st.append(v.strides[j])
                else:
                    return None
            return [0] * (4 - rank) + st, v.shape[-1] == D // 2

        tc, ts = table(cv), table(sv)
        if tc is None or tc != ts:
            return False
        t_st, half_table = tc
        pad = [0] * (4 - rank)
        x_st = pad + list(xv.strides[:-1])
        o_st = pad + list(contiguous_strides(tuple(xv.shape))[:-1])
        if any(s % vec for s in x_st + o_st) or any(s % t_align for s in t_st):
            return False
        if any((v.buf.base_off + v.offset * DTYPE_BYTES[v.buf.dtype]) % 16 for v in (xv, cv, sv)):
            return False
        bx, bc, bs = (self.based(v, n) for v, n in ((xv, x_val.name), (cv, c_val.name), (sv, s_val.name)))
        out = self.new_value_view(op.outputs[0])
        dims = [1] * (4 - rank) + list(xv.shape[:-1])
        p = N.RopeParams()
        p.batch, p.heads, p.rows, p.dim = dims[0], dims[1], dims[2], D
        p.x_sb, p.x_sh, p.x_sr = x_st
        p.o_sb, p.o_sh, p.o_sr = o_st
        p.t_sb, p.t_sh, p.t_sr = t_st
        p.half_table = int(half_table)
        p.x_dtype = N.DTYPE_CODE[dt]
        p.t_dtype = N.DTYPE_CODE[tdt]
        n = _prod(xv.shape)
        nbytes = 2 * n * DTYPE_BYTES[dt] + 2 * _prod(cv.shape) * tb  # x, out, and the two tables once
        self.emit(N.DP_K_ROPE, [bx.buf, bc.buf, bs.buf, out.buf], p, f"rope {tuple(xv.shape)} kernel",
                  6 * n, nbytes)
        return True

    def lower_attention_fused(self, op: Op, qv: View, qst, kv: View, kst, vv: View, vst, B, Hq, Hk, g, L, S, D,
                              Dv) -> None:
        """One fused tcgen05 attention record (scores stay on chip).  The query
        operand arrives as (view, (batch, head, row) strides); the output is
        token-major [B, L, H, Dv] for one query head per key head (so the usual
        transpose(1, 2).reshape that follows is free) and [B, H, L, Dv]
        otherwise (a group's heads stacked, as the kernel needs)."""
        out_v = op.outputs[0]
        p = N.AttentionParams()
        p.batch, p.heads_kv, p.group = B, Hk, g
        p.L, p.S, p.D, p.Dv = L, S, D, Dv
        p.q_sb, p.q_sh, p.q_sl = qst
        p.k_sb, p.k_sh, p.k_ss = kst[0], kst[1], kst[2]
        p.v_sb, p.v_sh, p.v_ss = vst[0], vst[1], vst[2]
        if g == 1 and len(out_v.type.shape) == 4:
            buf = self.new_buffer("arena", "bfloat16", (B, L, Hq, Dv), out_v.name)
            self.views[out_v.name] = View(buf, (B, Hq, L, Dv), (L * Hq * Dv, Dv, Hq * Dv, 1))
            p.o_sb, p.o_sh, p.o_sl = L * Hq * Dv, Dv, Hq * Dv
        else:
            buf = self.new_value_view(out_v).buf
            p.o_sb, p.o_sh, p.o_sl = Hq * L * Dv, L * Dv, Dv
        p.scale = float(op.attr("scale"))
        p.dtype = N.DP_BF16
        flops = 2 * B * Hq * L * S * (D + Dv)
        self.emit(N.DP_K_ATTENTION, [qv.buf, kv.buf, vv.buf, buf], p,
                  f"attention b{B} hkv{Hk} g{g} L{L} S{S} D{D} Dv{Dv}", flops,
                  qv.buf.nbytes + kv.buf.nbytes + vv.buf.nbytes + buf.nbytes)

    # ------------------------------------------------------------ embedding
    def lower_embedding(self, op: Op) -> None:
        ids = self.contiguous(op.inputs[0])
        w = self.contiguous(op.inputs[1])
        K = self.tf32_fold_width(op.outputs[0])
        src = self.views[op.inputs[1].name]
        if (K and src.buf.kind == "const" and src.buf.base is None and src.buf.name in self.const_tensors
                and w.buf is src.buf and w.buf.dtype == "float32" and len(w.shape) == 2):
            # Feeding a 3xTF32 linear: gather rows of the table split once at compile time.
            import torch
            name = src.buf.name + "|3xtf32rows"
            if name not in self.const_tensors:
                t = self.const_tensors[src.buf.name].float().reshape(w.shape)
                hi = (t.contiguous().view(torch.int32) & -8192).view(torch.float32)
                self.const_tensors[name] = torch.cat([hi, hi, t - hi], dim=1).contiguous()
            w = View(self.derived_const(name, "float32", (w.shape[0], 3 * K)), (w.shape[0], 3 * K), (3 * K, 1))
            out = self.new_tf32_split_view(op.outputs[0], K)
        else:
            out = self.new_value_view(op.outputs[0])
        p = N.EmbeddingParams()
        p.n_ids = _prod(ids.shape)
        p.vocab, p.dim = w.shape
        p.id_dtype = N.DTYPE_CODE[ids.buf.dtype]
        p.w_dtype = N.DTYPE_CODE[w.buf.dtype]
        self.emit(N.DP_K_EMBEDDING, [ids.buf, w.buf, out.buf], p, f"embedding {p.n_ids}x{p.dim}", 0,
                  ids.buf.nbytes + 2 * out.buf.nbytes)

    # -------------------------------------------------------------- regions
    def lower_region(self, op: Op) -> None:
        shape = materialized_shape(op.outputs[0])
        rb = RegionBuilder(shape)
        regs: Dict[str, int] = {}
        cur = op
        while True:
            r = self._emit_elementwise(rb, cur, regs)
            out_v = cur.outputs[0]
            regs[out_v.name] = r
            nxt = self.single_use(out_v)
            narrowing = cur.name == "to" and cur.attr("dtype") not in ("float32", "float64")
            if (nxt is None or id(nxt) in self.done or nxt.name not in ELEMENTWISE or nxt.name == "reshape"
                    or nxt.name == "transpose" or materialized_shape(nxt.outputs[0]) != shape or narrowing
                    or not rb.room()
                    or not all(v.name in regs or self.ready(v) for v in nxt.inputs if v is not out_v)):
                break
            self.done.add(id(nxt))
            cur = nxt
        out_v = cur.outputs[0]
        out = self.new_value_view(out_v)
        rb.store(out, regs[out_v.name])
        self.emit_region(rb, f"region {'+'.join(rb.names)} {shape}")

    def _emit_elementwise(self, rb: "RegionBuilder", op: Op, regs: Dict[str, int]) -> int:
        def operand(v: Value) -> int:
            if v.name in regs:
                return regs[v.name]
            return rb.load(self.views[v.name])

        rb.names.append(op.name)
        n = op.name
        if n in ELEMENTWISE_UNARY:
            return rb.unary(ELEMENTWISE_UNARY[n], operand(op.inputs[0]))
        if n == "gelu":
            return rb.unary("gelu_tanh" if op.attr("approximate") == "tanh" else "gelu_erf", operand(op.inputs[0]))
        if n in ELEMENTWISE_BINARY:
            return rb.binary(ELEMENTWISE_BINARY[n], operand(op.inputs[0]), operand(op.inputs[1]))
        if n in SCALAR_OPS:
            x = operand(op.inputs[0])
            c = rb.const(op.attr("scalar"))
            a, b = (c, x) if op.attr("reverse") else (x, c)
            return rb.binary(SCALAR_OPS[n], a, b)
        if n == "to":
            return rb.unary("mov", operand(op.inputs[0]))
        if n == "normalize":
            x = operand(op.inputs[0])
            if op.attr("mean") is None:
                return rb.unary("mov", x)
            cd = op.attr("channel_dim")
            m = rb.chansel(op.attr("mean"), cd)
            s = rb.chansel(op.attr("std"), cd)
            return rb.binary("div", rb.binary("sub", x, m), s)
        raise UnsupportedOpError(n)


class RegionBuilder:
    """Assembles one dp_region_desc: operands, registers, instructions."""

    def __init__(self, shape: Tuple[int, ...]):
        self.shape = tuple(shape) if shape else (1,)
        self.operands: List[Tuple[View, bool]] = []   # (view, is_output)
        self.instr: List[Tuple[str, int, int, int]] = []
        self.consts: List[float] = []
        self.nregs = 0
        self.chan_dims = set()
        self.names: List[str] = []
        self._loaded: Dict[Tuple, int] = {}
        # Registers holding an op's result (not a cached load): the chain
        # consumes each exactly once, so an instruction may overwrite one.
        self._temps = set()
        self._free: List[int] = []

    def room(self) -> bool:
        return (len(self.instr) < N.DP_REGION_MAX_INSTR - 8 and self.nregs < N.DP_REGION_MAX_REGS - 2
                and len(self.operands) < N.DP_REGION_MAX_OPERANDS - 2)

    def _reg(self) -> int:
        if self._free:
            return self._free.pop()
        r = self.nregs
        self.nregs += 1
        if self.nregs > N.DP_REGION_MAX_REGS:
            raise CompilationError("region: out of registers")
        return r

    def _result(self, *args: int) -> int:
        """Destination for an op reading ``args``: the first temporary among
        them (freed temporaries go back to the pool), else a new register."""
        temps = [a for a in dict.fromkeys(args) if a in self._temps]
        if temps:
            dst = temps[0]
            for t in temps[1:]:
                self._temps.discard(t)
                self._free.append(t)
            return dst
        r = self._reg()
        self._temps.add(r)
        return r

    def _bstrides(self, v: View) -> Tuple[int, ...]:
        """Strides of ``v`` broadcast to this region's shape."""
        rank = len(self.shape)
        vs = (1,) * (rank - len(v.shape)) + tuple(v.shape)
        st = (0,) * (rank - len(v.strides)) + tuple(v.strides)
        out = []
        for s_out, s_in, stv in zip(self.shape, vs, st):
            if s_in == s_out:
                out.append(stv if s_in != 1 else 0)
            elif s_in == 1:
                out.append(0)
            else:
                raise CompilationError(f"region: {v.shape} does not broadcast to {self.shape}")
        return tuple(out)

    def load(self, v: View) -> int:
        key = (id(v.buf), v.offset, tuple(v.shape), tuple(v.strides))
        if key in self._loaded:
            return self._loaded[key]
        self.operands.append((View(v.buf, v.shape, self._bstrides(v), v.offset), False))
        r = self._reg()
        self.instr.append(("load", r, len(self.operands) - 1, 0))
        self._loaded[key] = r
        return r

    def store(self, v: View, r: int) -> None:
        self.operands.append((View(v.buf, v.shape, self._bstrides(v), v.offset), True))
        self.instr.append(("store", 0, len(self.operands) - 1, r))

    def release(self, r: int) -> None:
        """Return temporary ``r`` (already stored) to the register pool."""
        if r in self._temps:
            self._temps.discard(r)
            self._free.append(r)

    def const(self, c: float) -> int:
        self.consts.append(float(c))
        r = self._reg()
        self._temps.add(r)
        self.instr.append(("const", r, len(self.consts) - 1, 0))
        return r

    def chansel(self, values, dim: int) -> int:
        base = len(self.consts)
        self.consts.extend(float(x) for x in values)
        if len(self.consts) > N.DP_REGION_MAX_CONST:
            raise CompilationError("region: too many per-channel constants")
        d = dim % len(self.shape)
        self.chan_dims.add(d)
        r = self._reg()
        self._temps.add(r)
        self.instr.append(("chansel", r, base, d))
        return r

    def unary(self, name: str, a: int) -> int:
        if name == "mov":  # a widening cast: the value is already a float in the register
            return a
        r = self._result(a)
        self.instr.append((name, r, a, 0))
        return r

    def binary(self, name: str, a: int, b: int) -> int:
        r = self._result(a, b)
        self.instr.append((name, r, a, b))
        return r

    def finish(self):
        # Inputs first, then outputs (the kernel's operand order).
        order = [i for i, (_, o) in enumerate(self.operands) if not o] + \
                [i for i, (_, o) in enumerate(self.operands) if o]
        remap = {old: new for new, old in enumerate(order)}
        n_in = sum(1 for _, o in self.operands if not o)
        shape, strides, dim_map = collapse_dims(self.shape, [self.operands[i][0].strides for i in order],
                                                self.chan_dims)
        d = N.RegionDesc()
        d.rank = len(shape)
        d.n_in = n_in
        d.n_out = len(self.operands) - n_in
        d.n_instr = len(self.instr)
        if d.n_instr > N.DP_REGION_MAX_INSTR:
            raise CompilationError("region: too many instructions")
        for k, s in enumerate(shape):
            d.shape[k] = s
        for new, old in enumerate(order):
            v = self.operands[old][0]
            d.dtype[new] = N.DTYPE_CODE[v.buf.dtype]
            d.offset[new] = v.offset
            for k in range(len(shape)):
                d.stride[new][k] = strides[new][k]
        for pc, (name, dst, a, b) in enumerate(self.instr):
            code = N.OP[name]
            if name in ("load", "store"):
                a = remap[a]
            if name == "chansel":
                b = dim_map[b]
            d.instr[pc] = code | (dst << 8) | (a << 16) | (b << 24)
        for i, c in enumerate(self.consts):
            d.consts[i] = c
        return d, [self.operands[i][0].buf for i in order]


def collapse_dims(shape, strides_list, keep):
    """Merge adjacent dims that every operand walks contiguously.

    Dims in ``keep`` (per-channel constant selectors) are never merged.
    Returns (shape, strides per operand, old-dim → new-dim map).
    """
    shape = list(shape)
    groups = [[0]]
    cur_shape = [shape[0]]
    cur_strides = [[s[0]] for s in strides_list]
    for i in range(1, len(shape)):
        mergeable = (i not in keep) and (groups[-1][-1] not in keep) and all(
            cs[-1] == s[i] * shape[i] for cs, s in zip(cur_strides, strides_list))
        if mergeable:
            groups[-1] = groups[-1] + [i]
            cur_shape[-1] *= shape[i]
            for cs, s in zip(cur_strides, strides_list):
                cs[-1] = s[i]
        else:
            groups.append([i])
            cur_shape.append(shape[i])
            for cs, s in zip(cur_strides, strides_list):
                cs.append(s[i])
    if len(cur_shape) > N.DP_REGION_MAX_RANK:
        raise CompilationError(f"region: rank {len(cur_shape)} after collapsing exceeds {N.DP_REGION_MAX_RANK}")
    dim_map = {}
    for new, g in enumerate(groups):
        for old in g:
            dim_map[old] = new
    return tuple(cur_shape), cur_strides, dim_map


def materialized_shape(v: Value) -> Tuple[int, ...]:
    """Shape stored for ``v``; a legacy scalar argmax stores one index per reduced row."""
    t = v.type
    if isinstance(t, TensorType):
        return t.shape if t.shape else (1,)
    if isinstance(t, ScalarType) and v.op is not None and v.op.name == "argmax":
        xt = v.op.inputs[0].type
        d = v.op.attr("dim") % len(xt.shape)
        shape = tuple(s for i, s in enumerate(xt.shape) if i != d)
        return shape if shape else (1,)
    raise CompilationError(f"value {v.name} of type {t!r} has no tensor storage")


def value_dtype(v: Value) -> str:
    return v.type.dtype


def plan_arena(buffers: List[Buffer]) -> int:
    """First-fit offsets for arena buffers whose live ranges overlap in time;
    a sub-range slot sits at its root's offset plus its own."""
    arena = [b for b in buffers if b.kind == "arena" and b.base is None]
    for b in arena:
        if b.first < 0:  # produced but never used: keep it alive at its producer only
            b.first = b.last = 0
    placed: List[Buffer] = []
    top = 0
    for b in sorted(arena, key=lambda x: (-x.nbytes, x.first)):
        size = _round(b.nbytes)
        busy = sorted((p.offset, p.offset + _round(p.nbytes)) for p in placed
                      if not (p.last < b.first or b.last < p.first))
        off = 0
        for lo, hi in busy:
            if off + size <= lo:
                break
            off = max(off, hi)
        b.offset = off
        placed.append(b)
        top = max(top, off + size)
    for b in buffers:
        if b.base is not None and b.root.kind == "arena":
            b.offset = b.root.offset + b.base_off
    return top


def _round(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def lower(fn: Function, const_names=(), const_tensors=None) -> Lowered:
    """Lower ``fn``.  With ``const_tensors`` (the constants' values) the
    lowering may also derive new constants, e.g. the concatenated weight of
    sibling linears; they are returned in ``Lowered.extra_consts``."""
    return Lowerer(fn, const_names, const_tensors).run()
