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
        self._checks_index = any(r["kernel"] == "embedding" for r in spec.records)

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
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"input {io.name}: expected a torch.Tensor, got {type(t).__name__}")
        if t.numel() != io.numel:
            raise N.DevProcError(N.DP_ERR_SHAPE, f"input {io.name}: shape {tuple(t.shape)} does not match "
                                                 f"the compiled shape {tuple(io.shape)}")
        if t.dtype != want:
            raise N.DevProcError(N.DP_ERR_SHAPE, f"input {io.name}: dtype {t.dtype} != compiled {want}")
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

    def run(self, *args, to_cpu: bool = True, reuse_host_buffers: bool = False, **kwargs) -> List[torch.Tensor]:
        """Execute once.  Inputs by IR name (positional args fill the inputs in
        order).  Returns fresh CPU tensors (``to_cpu=True``, the reference's
        behaviour); with ``reuse_host_buffers`` the program's pinned host
        output buffers themselves (no host copy; the next run overwrites
        them); with ``to_cpu=False`` the device output buffers (likewise
        overwritten by the next run)."""
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
                self._bind_input(io, given[io.name])
            stream = torch.cuda.current_stream(self._device())
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
            if self._checks_index:
                code, info = N.device_error()
                if code == N.DP_DEVERR_INDEX:
                    raise IndexError(f"embedding id out of range at flat position {info}")
                if code != N.DP_DEVERR_NONE:
                    raise N.DevProcError(N.DP_ERR_DEVICE, f"device error {code} (info {info})")
            return outs if reuse_host_buffers else [h.clone() for h in outs]

    def __call__(self, *args, **kwargs):
        return self.run(*args, **kwargs)

    # ------------------------------------------------------- persistence
    def export(self, path: str) -> None:
        path = str(path)
        with open(path, "wb") as f:
            f.write(self.spec.plan)
        offset = 0
        consts = []
        if self.spec.consts:
            with open(path + ".weights", "wb") as f:
                for c in self.spec.consts:
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
            "outputs": [asdict(o) for o in self.spec.outputs],
            "kernels": self.spec.records,
            "aliases": self.spec.aliases,
            "tensor_allocations": {o.name: {"shape": o.shape, "dtype": o.dtype} for o in self.spec.outputs},
        }
        with open(path + ".meta.json", "w") as f:
            json.dump(meta, f, indent=1)

    @staticmethod
    def load(path: str, device_id: int = 0) -> "B200CompiledProgram":
        path = str(path)
        with open(path + ".meta.json") as f:
            meta = json.load(f)
        if meta.get("format") != FORMAT or meta.get("version") != FORMAT_VERSION:
            raise ValueError(f"{path}: not a {FORMAT} v{FORMAT_VERSION} program")
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
        spec = ProgramSpec(meta["name"], plan, [IOSlot(**i) for i in meta["inputs"]], consts,
                           [IOSlot(**o) for o in meta["outputs"]], meta["arena_bytes"], meta["kernels"],
                           meta.get("aliases", []))
        return B200CompiledProgram(spec, constants, device_id)

    def close(self) -> None:
        if self._native is not None:
            self._native.close()
            self._native = None

    def describe(self) -> str:
        lines = [f"program {self.spec.name}: {len(self.spec.records)} launches, arena "
                 f"{self.spec.arena_bytes / 2**20:.1f} MiB"]
        lines += [f"  [{i}] {r['label']}" for i, r in enumerate(self.spec.records)]
        return "\n".join(lines)
