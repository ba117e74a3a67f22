"""A compiled program with host steps around its GPU plan.

``B200Compiler.compile`` returns this when the function has tokenizer,
string or dict ops (``backend/host_ops.py``): the host prologue runs on the
CPU with the reference's CPU-backend semantics, its tensors (token ids) feed
the device plan, and the host epilogue (e.g. decoding argmax ids back to
text) reads the plan's results.  Inputs are keyword arguments named after
the IR inputs as for any program: tensors, and Python ``str`` for string
inputs.  ``export`` writes the device plan as usual and records the host
steps in ``<path>.meta.json``; ``load`` restores both.
"""

import json
from typing import Any, Dict, List, Optional

import torch

from ..base import CompiledProgram
from ..host_ops import TokenizerCache, run_host_op


class _Named:
    def __init__(self, name: str):
        self.name = name


class HostOpRecord:
    """A host op as stored in a saved program: name, value names, attributes."""

    def __init__(self, name: str, inputs: List[str], outputs: List[str], attrs: Dict[str, Any]):
        self.name = name
        self.inputs = [_Named(n) for n in inputs]
        self.outputs = [_Named(n) for n in outputs]
        self.attrs = dict(attrs)

    @staticmethod
    def of(op) -> "HostOpRecord":
        return HostOpRecord(op.name, [v.name for v in op.inputs], [v.name for v in op.outputs], dict(op.attrs))

    def to_json(self) -> Dict[str, Any]:
        return {"name": self.name, "inputs": [v.name for v in self.inputs],
                "outputs": [v.name for v in self.outputs], "attrs": self.attrs}


class HostDeviceProgram(CompiledProgram):
    """Host prologue → device plan → host epilogue."""

    def __init__(self, input_names: List[str], output_names: List[str], prologue: List[HostOpRecord],
                 device, epilogue: List[HostOpRecord], device_inputs: List[str], device_outputs: List[str],
                 ir_function=None):
        self._input_names = list(input_names)
        self._output_names = list(output_names)
        self.prologue = list(prologue)
        self.device = device  # a B200CompiledProgram, or None for a host-only function
        self.epilogue = list(epilogue)
        self.device_inputs = list(device_inputs)
        self.device_outputs = list(device_outputs)
        self.ir_function = ir_function
        self.tokenizers = TokenizerCache()

    @staticmethod
    def from_split(fn, prologue, device, epilogue, device_inputs, device_outputs) -> "HostDeviceProgram":
        return HostDeviceProgram([v.name for v in fn.inputs if v.name not in (getattr(fn, "constants", None) or {})],
                                 [v.name for v in fn.outputs], [HostOpRecord.of(o) for o in prologue], device,
                                 [HostOpRecord.of(o) for o in epilogue], device_inputs, device_outputs, fn)

    @property
    def input_names(self) -> List[str]:
        return list(self._input_names)

    @property
    def output_names(self) -> List[str]:
        return list(self._output_names)

    @property
    def spec(self):
        return self.device.spec if self.device is not None else None

    def run(self, *args, to_cpu: bool = True, **kwargs) -> List[Any]:
        if len(args) > len(self._input_names):
            raise TypeError(f"{len(args)} positional inputs for {len(self._input_names)} program inputs")
        env: Dict[str, Any] = dict(zip(self._input_names, args))
        for k, v in kwargs.items():
            if k in env:
                raise TypeError(f"input {k} given twice")
            env[k] = v
        missing = [n for n in self._input_names if n not in env]
        if missing:
            raise TypeError(f"missing inputs {missing}")
        for op in self.prologue:
            run_host_op(op, env, self.tokenizers)
        if self.device is not None:
            feed = {n: env[n] for n in self.device.input_names}
            host_results = to_cpu or bool(self.epilogue)
            outs = self.device.run(**feed, to_cpu=host_results)
            env.update(zip(self.device.output_names, outs))
        for op in self.epilogue:
            run_host_op(op, env, self.tokenizers)
        return [env[n] for n in self._output_names]

    def __call__(self, *args, **kwargs):
        return self.run(*args, **kwargs)

    def synchronize(self) -> None:
        if self.device is not None:
            self.device.synchronize()

    def host_meta(self) -> Dict[str, Any]:
        return {"inputs": self._input_names, "outputs": self._output_names,
                "prologue": [o.to_json() for o in self.prologue], "epilogue": [o.to_json() for o in self.epilogue],
                "device_inputs": self.device_inputs, "device_outputs": self.device_outputs,
                "has_device": self.device is not None}

    def export(self, path: str) -> None:
        from .program import FORMAT, FORMAT_VERSION
        path = str(path)
        if self.device is not None:
            self.device.export(path)
            with open(path + ".meta.json") as f:
                meta = json.load(f)
        else:
            meta = {"format": FORMAT, "version": FORMAT_VERSION, "name": "host"}
        meta["host"] = self.host_meta()
        with open(path + ".meta.json", "w") as f:
            json.dump(meta, f, indent=1)

    @staticmethod
    def from_meta(path: str, meta: Dict[str, Any], device_id: int = 0) -> "HostDeviceProgram":
        from .program import B200CompiledProgram
        h = meta["host"]
        device = B200CompiledProgram.load(path, device_id, host_ok=False) if h["has_device"] else None
        rec = lambda d: HostOpRecord(d["name"], d["inputs"], d["outputs"], d["attrs"])  # noqa: E731
        return HostDeviceProgram(h["inputs"], h["outputs"], [rec(d) for d in h["prologue"]], device,
                                 [rec(d) for d in h["epilogue"]], h["device_inputs"], h["device_outputs"])

    @staticmethod
    def load(path: str, device_id: int = 0) -> "HostDeviceProgram":
        with open(str(path) + ".meta.json") as f:
            meta = json.load(f)
        return HostDeviceProgram.from_meta(str(path), meta, device_id)

    def close(self) -> None:
        if self.device is not None:
            self.device.close()
