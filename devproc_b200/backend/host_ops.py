"""Host steps of a compiled program: tokenizer, string and dict ops.

These ops are not data-parallel GPU work; the reference executes them on the
host with its CPU backend (src/devproc/backend/cpu/ops.py:24-251, dispatched
by ``handle_op`` :253-262), and so does this backend.  ``split_host_ops``
cuts a function into a host prologue (host ops that need no device result),
the device body (every tensor op, compiled to one GPU plan) and a host
epilogue (host ops that read device results, e.g. decoding argmax ids), and
``HostDeviceProgram`` runs the three in order.  Each handler keeps the
reference's semantics:

* ``load_tokenizer``: the handle is the tokenizer path; the tokenizer is
  loaded on first use with ``transformers.AutoTokenizer.from_pretrained`` and
  cached per path (cpu/codegen.py:63-71, without its silent ``None`` on a
  failed load: a missing tokenizer raises);
* ``tokenize_encode``: ``tokenizer.encode(text, max_length=2048,
  truncation=True, padding="max_length")`` as int32 (ops.py:38-64);
* ``tokenize_decode``: ids without the pad id, then ``tokenizer.decode``
  (ops.py:67-86);
* ``string_length`` / ``string_concat`` / ``string_slice``: ``len``, ``+``,
  ``text[start:end]`` (ops.py:91-139); ``string_format`` returns its template
  unchanged, as the reference does (ops.py:142-154);
* ``dict_create`` / ``dict_get`` / ``dict_set`` / ``dict_size``: a Python dict
  of tensors keyed by string; ``dict_set`` stores a clone (ops.py:159-218).
  ``dict_get`` of a missing key raises KeyError (the reference left the value
  unset, so its next use failed).
"""

from typing import Any, Dict, List, Optional, Tuple

import torch

from ..ir.function import Function
from ..ir.types import TensorType

HOST_OP_NAMES = ("load_tokenizer", "tokenize_encode", "tokenize_decode", "string_length", "string_concat",
                 "string_slice", "string_format", "dict_create", "dict_get", "dict_set", "dict_size")


class TokenizerCache:
    """Tokenizers by path, loaded once."""

    def __init__(self):
        self._by_path: Dict[str, Any] = {}

    def get(self, path: str):
        tok = self._by_path.get(path)
        if tok is None:
            try:
                from transformers import AutoTokenizer
            except ImportError as e:
                raise RuntimeError("tokenizer ops need the transformers package") from e
            tok = AutoTokenizer.from_pretrained(path)
            self._by_path[path] = tok
        return tok


def _attr(op, name, default=None):
    return op.attrs.get(name, default)


def run_host_op(op, env: Dict[str, Any], tokenizers: TokenizerCache) -> None:
    """Execute one host op, reading its inputs from and writing its output to ``env``."""
    n = op.name
    ins = [env[v.name] for v in op.inputs]
    out = op.outputs[0].name if op.outputs else None
    if n == "load_tokenizer":
        env[out] = _attr(op, "tokenizer_path")
    elif n == "tokenize_encode":
        tok = tokenizers.get(ins[0])
        ids = tok.encode(ins[1], max_length=_attr(op, "max_length", 2048), truncation=True, padding="max_length")
        env[out] = torch.tensor(ids, dtype=torch.int32)
    elif n == "tokenize_decode":
        tok = tokenizers.get(ins[0])
        ids = ins[1].reshape(-1).tolist()
        if tok.pad_token_id is not None:
            ids = [t for t in ids if t != tok.pad_token_id]
        env[out] = tok.decode(ids)
    elif n == "string_length":
        env[out] = torch.tensor(len(ins[0]), dtype=torch.int32)
    elif n == "string_concat":
        env[out] = ins[0] + ins[1]
    elif n == "string_slice":
        env[out] = ins[0][_attr(op, "start", 0):_attr(op, "end")]
    elif n == "string_format":
        env[out] = ins[0]
    elif n == "dict_create":
        env[out] = {}
    elif n == "dict_get":
        if ins[1] not in ins[0]:
            raise KeyError(f"dict_get: key {ins[1]!r} not in the dict")
        env[out] = ins[0][ins[1]]
    elif n == "dict_set":
        ins[0][ins[1]] = ins[2].clone()
        env[out] = ins[0]
    elif n == "dict_size":
        env[out] = torch.tensor(len(ins[0]), dtype=torch.int32)
    else:
        raise NotImplementedError(f"host op '{n}'")


def split_host_ops(fn: Function) -> Optional[Tuple[list, Function, list, List[str], List[str]]]:
    """(prologue ops, device Function, epilogue ops, device input names,
    device output names), or None when ``fn`` has no host op.

    The device Function has the tensor ops in order; its inputs are the
    function's tensor inputs and the prologue's tensors that device ops read,
    its outputs the device values the epilogue reads or the function returns.
    A device op that reads an epilogue value would need a second device
    segment and is rejected."""
    from .base import CompilationError
    ops = list(fn.block.ops)
    if not any(op.name in HOST_OP_NAMES for op in ops):
        return None
    host_avail = {v.name for v in fn.inputs}  # values known before the device body runs
    dev_made = set()
    prologue, device, epilogue = [], [], []
    for op in ops:
        reads = [v.name for v in op.inputs]
        if op.name in HOST_OP_NAMES:
            if all(r in host_avail for r in reads):
                prologue.append(op)
                host_avail.update(v.name for v in op.outputs)
            else:
                epilogue.append(op)
        else:
            epi_out = {v.name for e in epilogue for v in e.outputs}
            if any(r in epi_out for r in reads):
                raise CompilationError(f"op '{op.name}' reads a host value computed from device results; "
                                       "a program has one device segment")
            device.append(op)
            dev_made.update(v.name for v in op.outputs)
    by_name = {v.name: v for v in fn.inputs}
    for op in ops:
        for v in op.outputs:
            by_name[v.name] = v
    dev_reads = []
    for op in device:
        for v in op.inputs:
            if v.name not in dev_made and v.name not in dev_reads:
                dev_reads.append(v.name)
    for name in dev_reads:
        if not isinstance(by_name[name].type, TensorType):
            raise CompilationError(f"device op reads host value {name} ({by_name[name].type!r})")
    wanted = [v.name for e in epilogue for v in e.inputs] + [v.name for v in fn.outputs]
    dev_out = []
    for name in wanted:
        if name in dev_made and name not in dev_out:
            dev_out.append(name)
    sub = Function(fn.name + "_device")
    for name in dev_reads:
        sub.add_input(by_name[name])
    for op in device:
        sub.add_op(op)
    sub.outputs = [by_name[n] for n in dev_out]
    consts = getattr(fn, "constants", None)
    if consts:
        sub.constants = {k: v for k, v in consts.items() if k in dev_reads}
    return prologue, sub, epilogue, dev_reads, dev_out
