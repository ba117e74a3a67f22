"""Compiled program: a validated plan, a static arena and persistent I/O buffers.

``run`` keeps the reference's calling convention (keyword inputs named after
the IR inputs, a list of output tensors back, CPU tensors by default —
src/devproc/backend/triton/compiler.py:54-68, 189-250) but allocates nothing
on the device per call: constants (weights) are uploaded once, outputs and
input staging buffers are allocated once, intermediates live in the arena
the native program owns, and the launch sequence is replayed as one CUDA
graph after the first run.

``export`` writes ``path`` (the binary plan), ``path.meta.json`` (I/O tables,
records, arena size — the reference's meta file name, serialization.py:
165-233) and, when the program has constants, ``path.weights``.  ``load``
rebuilds a runnable program from those files alone; no IR is needed.
"""

import json
import os
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional

import torch

from ... import _native as N
from ..base import CompiledProgram

FORMAT = "devproc-b200-program"
FORMAT_VERSION = 1

TORCH_DTYPES = {"uint8": torch.uint8, "int8": torch.int8, "int16": torch.int16, "int32": torch.int32,
                "int64": torch.int64, "float16": torch.float16, "bfloat16": torch.bfloat16,
                "float32": torch.float32, "float64": torch.float64, "bool": torch.bool}


@dataclass
class IOSlot:
    name: str
    slot: int
    shape: List[int]
    dtype: str
    offset: int = 0  # byte offset in the weights file (constants only)

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


@dataclass
class ProgramSpec:
    name: str
    plan: bytes
    inputs: List[IOSlot]
    consts: List[IOSlot]
    outputs: List[IOSlot]
    arena_bytes: int
    records: List[Dict[str, Any]] = field(default_factory=list)
    # caller-bound slots that name a byte range of another slot's buffer:
    # [slot, root slot, byte offset]; bound at the root's pointer + offset
    aliases: List[List[int]] = field(default_factory=list)

    @staticmethod
    def from_lowered(low) -> "ProgramSpec":
        def io(pairs):
            return [IOSlot(n, b.slot, list(b.shape), b.dtype) for n, b in pairs]
        recs = [{"kernel": N.KERNEL_NAMES[r.kernel], "label": r.label, "flops": r.flops, "bytes": r.bytes}
                for r in low.records]
        return ProgramSpec(low.name, low.plan_bytes(), io(low.inputs), io(low.consts), io(low.outputs),
                           low.arena_bytes, recs, [list(a) for a in low.aliases])


class B200CompiledProgram(CompiledProgram):
    """A compiled DevProc program running on the sm_100a C-ABI library."""

    def __init__(self, spec: ProgramSpec, constants: Optional[Dict[str, torch.Tensor]] = None,
                 device_id: int = 0, ir_function=None, use_graph: bool = True):
        self.spec = spec
        self.device_id = device_id
        self.ir_function = ir_function
        self.use_graph = use_graph
        self._constants = dict(constants or {})
        missing = [c.name for c in spec.consts if c.name not in self._constants]
        if missing:
            raise ValueError(f"constants missing for {missing}")
        self._native: Optional[N.NativeProgram] = None
        self._dev_consts: Dict[str, torch.Tensor] = {}
        self._outputs: List[torch.Tensor] = []
        self._staging: Dict[str, torch.Tensor] = {}
        self._host_out: List[Optional[torch.Tensor]] = []
        self._bound: Dict[int, int] = {}
        # chunked execution for host inputs (see set_stream)
        self.stream_chunk: Optional[int] = None
        self._chunk: Optional["B200CompiledProgram"] = None
        self._side: Optional[tuple] = None

    # reference-compatible attributes ----------------------------------
    @property
    def tensor_allocations(self) -> Dict[str, Any]:
        return {o.name: (tuple(o.shape), o.dtype) for o in self.spec.outputs}

    @property
    def input_names(self) -> List[str]:
        return [i.name for i in self.spec.inputs]

    @property
    def output_names(self) -> List[str]:
        return [o.name for o in self.spec.outputs]

    @property
    def kernels(self) -> List[Dict[str, Any]]:
        return list(self.spec.records)

    # -------------------------------------------------------------------
    def _device(self) -> torch.device:
        return torch.device("cuda", self.device_id)

    def _ensure_ready(self) -> None:
        if self._native is not None:
            return
        if not torch.cuda.is_available():
            raise N.DevProcError(N.DP_ERR_STATE, "no CUDA device visible: the B200 backend has no CPU "
                                                 "execution path")
        N.device_init(self.device_id)
        dev = self._device()
        with torch.cuda.device(dev):
            prog = N.NativeProgram(self.spec.plan, self.device_id)
            for c in self.spec.consts:
                # one device copy per constant; it stays referenced for as long as a slot points at it
                t = self._dev_consts.get(c.name)
                if t is None:
                    t = self._constants[c.name]
                    t = t.detach().to(device=dev, dtype=TORCH_DTYPES[c.dtype]).contiguous()
                    self._dev_consts[c.name] = t
                if list(t.shape) != list(c.shape):
                    raise N.DevProcError(N.DP_ERR_SHAPE, f"constant {c.name}: shape {tuple(t.shape)} != "
                                                         f"{tuple(c.shape)}")
                self._bind_slot(prog, c.slot, t.data_ptr(), t.numel() * t.element_size())
            for o in self.spec.outputs:
                t = torch.empty(o.shape, dtype=TORCH_DTYPES[o.dtype], device=dev)
                self._outputs.append(t)
                self._bind_slot(prog, o.slot, t.data_ptr(), max(1, t.numel()) * t.element_size())
            prog.set_graph(self.use_graph)
            self._host_out = [None] * len(self._outputs)
        self._native = prog

    def _bind_slot(self, prog, slot: int, ptr: int, nbytes: int) -> None:
        """Bind ``slot`` and every slot that names a byte range of it."""
        prog.bind(slot, ptr, nbytes)
        for a, root, off in self.spec.aliases:
            if root == slot:
                prog.bind(a, ptr + off, nbytes - off)

    def _bind_input(self, io: IOSlot, t: torch.Tensor) -> None:
        want = TORCH_DTYPES[io.dtype]
        t = self._check_input(io, t)
        dev = self._device()
        if t.is_cuda and t.device == dev and t.is_contiguous():
            src = t
        else:
            st = self._staging.get(io.name)
            if st is None:
                st = torch.empty(io.shape, dtype=want, device=dev)
                self._staging[io.name] = st
            st.view(-1).copy_(t.reshape(-1), non_blocking=True)
            src = st
        ptr = src.data_ptr()
        if self._bound.get(io.slot) != ptr:
            self._bind_slot(self._native, io.slot, ptr, max(1, src.numel()) * src.element_size())
            self._bound[io.slot] = ptr

    def clone(self) -> "B200CompiledProgram":
        """The same plan and constants with its own arena and output buffers;
        the device copies of the constants are shared, not uploaded again."""
        c = B200CompiledProgram(self.spec, self._constants, self.device_id, self.ir_function, self.use_graph)
        c._dev_consts = self._dev_consts
        if self._chunk is not None:
            c.set_stream(self.stream_chunk, self._chunk.spec)
        return c

    def set_stream(self, chunk: int, chunk_spec: ProgramSpec) -> None:
        """Attach the same program compiled for a batch of ``chunk`` samples.
        ``run`` with host inputs then executes it on successive chunks of the
        batch: chunk i+1's inputs cross PCIe on one stream while chunk i runs
        and chunk i-1's outputs come back on another, instead of one whole
        copy in, the launches, and one whole copy out."""
        batch = self.spec.inputs[0].shape[0]
        if batch % chunk or chunk_spec.inputs[0].shape[0] != chunk:
            raise ValueError(f"chunk {chunk} does not divide batch {batch}")
        self.stream_chunk = chunk
        self._chunk = B200CompiledProgram(chunk_spec, self._constants, self.device_id, use_graph=False)
        self._chunk._dev_consts = self._dev_consts  # one upload per constant, shared

    def _run_streamed(self, given: Dict[str, torch.Tensor], to_cpu: bool) -> List[torch.Tensor]:
        sub = self._chunk
        sub._ensure_ready()
        dev = self._device()
        cur = torch.cuda.current_stream(dev)
        if self._side is None:
            self._side = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        h2d, d2h = self._side
        batch, b = self.spec.inputs[0].shape[0], self.stream_chunk
        start = torch.cuda.Event()
        start.record(cur)
        h2d.wait_event(start)
        rows = []  # (chunk IOSlot, full-batch source [batch, -1], host source or None)
        for io, cio in zip(self.spec.inputs, sub.spec.inputs):
            t = self._check_input(io, given[io.name])
            if t.is_cuda and t.device == dev and t.is_contiguous():
                rows.append((cio, t.view(batch, -1), None))
                continue
            st = self._staging.get(io.name)
            if st is None:
                st = torch.empty(io.shape, dtype=t.dtype, device=dev)
                self._staging[io.name] = st
            rows.append((cio, st.view(batch, -1), t.reshape(batch, -1)))
        outs = [o.view(batch, -1) for o in self._outputs]
        host = []
        if to_cpu:
            d2h.wait_event(start)
            for i, t in enumerate(self._outputs):
                if self._host_out[i] is None:
                    self._host_out[i] = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                host.append(self._host_out[i].view(batch, -1))
        for i in range(batch // b):
            lo, hi = i * b, (i + 1) * b
            staged = torch.cuda.Event()
            with torch.cuda.stream(h2d):
                for _, dst, src in rows:
                    if src is not None:
                        dst[lo:hi].copy_(src[lo:hi], non_blocking=True)
                staged.record(h2d)
            cur.wait_event(staged)
            for cio, dst, _ in rows:
                part = dst[lo:hi]
                sub._bind_slot(sub._native, cio.slot, part.data_ptr(), max(1, part.numel()) * part.element_size())
            for cio, o in zip(sub.spec.outputs, outs):
                part = o[lo:hi]
                sub._bind_slot(sub._native, cio.slot, part.data_ptr(), max(1, part.numel()) * part.element_size())
            sub._native.run(cur.cuda_stream)
            if to_cpu:
                done = torch.cuda.Event()
                done.record(cur)
                d2h.wait_event(done)
                with torch.cuda.stream(d2h):
                    for h, o in zip(host, outs):
                        h[lo:hi].copy_(o[lo:hi], non_blocking=True)
        if to_cpu:
            back = torch.cuda.Event()
            back.record(d2h)
            cur.wait_event(back)
        return [self._host_out[i] for i in range(len(outs))] if to_cpu else list(self._outputs)

    def _check_input(self, io: IOSlot, t) -> torch.Tensor:
        want = TORCH_DTYPES[io.dtype]
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"input {io.name}: expected a torch.Tensor, got {type(t).__name__}")
        if t.numel() != io.numel:
            raise N.DevProcError(N.DP_ERR_SHAPE, f"input {io.name}: shape {tuple(t.shape)} does not match "
                                                 f"the compiled shape {tuple(io.shape)}")
        if t.dtype != want:
            raise N.DevProcError(N.DP_ERR_SHAPE, f"input {io.name}: dtype {t.dtype} != compiled {want}")
        return t

    def run(self, *args, to_cpu: bool = True, reuse_host_buffers: bool = False, **kwargs) -> List[torch.Tensor]:
        """Execute once.  Inputs by IR name (positional args fill the inputs in
        order).  Returns fresh CPU tensors (``to_cpu=True``, the reference's
        behaviour); with ``reuse_host_buffers`` the program's pinned host
        output buffers themselves (no host copy; the next run overwrites
        them); with ``to_cpu=False`` the device output buffers (likewise
        overwritten by the next run), enqueued without waiting.

        A run that returns host tensors synchronises and then raises if a
        kernel reported an error through the device error word: IndexError
        for an embedding id out of range, DevProcError (DP_ERR_DEVICE) for a
        bounded wait that gave up.  After ``to_cpu=False`` runs,
        ``synchronize()`` does the same check."""
        self._ensure_ready()
        if len(args) > len(self.spec.inputs):
            raise TypeError(f"{len(args)} positional inputs for {len(self.spec.inputs)} program inputs")
        given = dict(zip([i.name for i in self.spec.inputs], args))
        for k, v in kwargs.items():
            if k in given:
                raise TypeError(f"input {k} given twice")
            given[k] = v
        unknown = set(given) - {i.name for i in self.spec.inputs}
        if unknown:
            raise TypeError(f"unknown inputs {sorted(unknown)}; program inputs are {self.input_names}")
        with torch.cuda.device(self._device()):
            for io in self.spec.inputs:
                if io.name not in given:
                    raise TypeError(f"missing input {io.name}")
            stream = torch.cuda.current_stream(self._device())
            if self._chunk is not None and any(not given[io.name].is_cuda for io in self.spec.inputs
                                               if isinstance(given[io.name], torch.Tensor)):
                outs = self._run_streamed(given, to_cpu)
                if not to_cpu:
                    return outs
            else:
                for io in self.spec.inputs:
                    self._bind_input(io, given[io.name])
                self._native.run(stream.cuda_stream)
                if not to_cpu:
                    return list(self._outputs)
                outs = []
                for i, t in enumerate(self._outputs):
                    h = self._host_out[i]
                    if h is None:
                        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                        self._host_out[i] = h
                    h.copy_(t, non_blocking=True)
                    outs.append(h)
            stream.synchronize()
            N.raise_device_error(self.device_id, f"program {self.spec.name}")
            return outs if reuse_host_buffers else [h.clone() for h in outs]

    def synchronize(self) -> None:
        """Wait for the work ``run(to_cpu=False)`` enqueued on the current
        stream and raise if one of its kernels reported an error (an embedding
        id out of range, a bounded wait that gave up).  ``run`` with host
        results does this itself after every call."""
        with torch.cuda.device(self._device()):
            torch.cuda.current_stream(self._device()).synchronize()
        N.raise_device_error(self.device_id, f"program {self.spec.name}")

    def __call__(self, *args, **kwargs):
        return self.run(*args, **kwargs)

    # ------------------------------------------------------- persistence
    def export(self, path: str) -> None:
        path = str(path)
        with open(path, "wb") as f:
            f.write(self.spec.plan)
        offset = 0
        consts = []
        to_write = list(self.spec.consts)
        if self._chunk is not None:
            have = {c.name for c in to_write}
            to_write += [c for c in self._chunk.spec.consts if c.name not in have]
        if to_write:
            with open(path + ".weights", "wb") as f:
                for c in to_write:
                    t = self._constants[c.name].detach().to("cpu", TORCH_DTYPES[c.dtype]).contiguous()
                    raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
                    pad = (-offset) % 256
                    f.write(b"\0" * pad)
                    offset += pad
                    consts.append(IOSlot(c.name, c.slot, c.shape, c.dtype, offset))
                    f.write(raw)
                    offset += len(raw)
        meta = {
            "format": FORMAT, "version": FORMAT_VERSION, "name": self.spec.name, "device_id": self.device_id,
            "plan_bytes": len(self.spec.plan), "arena_bytes": self.spec.arena_bytes,
            "inputs": [asdict(i) for i in self.spec.inputs],
            "consts": [asdict(c) for c in consts],
            "n_consts": len(self.spec.consts),
            "outputs": [asdict(o) for o in self.spec.outputs],
            "kernels": self.spec.records,
            "aliases": self.spec.aliases,
            "tensor_allocations": {o.name: {"shape": o.shape, "dtype": o.dtype} for o in self.spec.outputs},
        }
        if self._chunk is not None:
            cs = self._chunk.spec
            with open(path + ".chunk", "wb") as f:
                f.write(cs.plan)
            meta["stream"] = {"chunk": self.stream_chunk, "plan_bytes": len(cs.plan), "arena_bytes": cs.arena_bytes,
                              "inputs": [asdict(i) for i in cs.inputs], "consts": [asdict(c) for c in cs.consts],
                              "outputs": [asdict(o) for o in cs.outputs], "kernels": cs.records,
                              "aliases": cs.aliases}
        with open(path + ".meta.json", "w") as f:
            json.dump(meta, f, indent=1)

    @staticmethod
    def load(path: str, device_id: int = 0, host_ok: bool = True):
        """Rebuild a saved program; one saved with host steps (tokenizer, string
        or dict ops) comes back as a HostDeviceProgram around its device plan."""
        path = str(path)
        with open(path + ".meta.json") as f:
            meta = json.load(f)
        if meta.get("format") != FORMAT or meta.get("version") != FORMAT_VERSION:
            raise ValueError(f"{path}: not a {FORMAT} v{FORMAT_VERSION} program")
        if host_ok and "host" in meta:
            from .host_program import HostDeviceProgram
            return HostDeviceProgram.from_meta(path, meta, device_id)
        with open(path, "rb") as f:
            plan = f.read()
        if len(plan) != meta["plan_bytes"]:
            raise ValueError(f"{path}: plan size {len(plan)} != {meta['plan_bytes']}")
        consts = [IOSlot(**c) for c in meta["consts"]]
        constants = {}
        if consts:
            blob = open(path + ".weights", "rb").read()
            for c in consts:
                nbytes = c.numel * torch.empty((), dtype=TORCH_DTYPES[c.dtype]).element_size()
                raw = bytearray(blob[c.offset:c.offset + nbytes])
                t = torch.frombuffer(raw, dtype=torch.uint8) if nbytes else torch.empty(0, dtype=torch.uint8)
                constants[c.name] = t.view(TORCH_DTYPES[c.dtype]).reshape(c.shape)
        # the weights file may also hold constants only the chunk program reads (after the first n_consts)
        spec = ProgramSpec(meta["name"], plan, [IOSlot(**i) for i in meta["inputs"]],
                           consts[:meta.get("n_consts", len(consts))],
                           [IOSlot(**o) for o in meta["outputs"]], meta["arena_bytes"], meta["kernels"],
                           meta.get("aliases", []))
        prog = B200CompiledProgram(spec, constants, device_id)
        st = meta.get("stream")
        if st:
            with open(path + ".chunk", "rb") as f:
                cplan = f.read()
            if len(cplan) != st["plan_bytes"]:
                raise ValueError(f"{path}.chunk: plan size {len(cplan)} != {st['plan_bytes']}")
            prog.set_stream(st["chunk"], ProgramSpec(meta["name"], cplan, [IOSlot(**i) for i in st["inputs"]],
                                                     [IOSlot(**c) for c in st["consts"]],
                                                     [IOSlot(**o) for o in st["outputs"]], st["arena_bytes"],
                                                     st["kernels"], st.get("aliases", [])))
        return prog

    def close(self) -> None:
        if self._native is not None:
            self._native.close()
            self._native = None

    def describe(self) -> str:
        lines = [f"program {self.spec.name}: {len(self.spec.records)} launches, arena "
                 f"{self.spec.arena_bytes / 2**20:.1f} MiB"]
        lines += [f"  [{i}] {r['label']}" for i, r in enumerate(self.spec.records)]
        return "\n".join(lines)
