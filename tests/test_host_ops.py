"""Host tokenizer / string / dict steps (no GPU needed).

The handlers in ``devproc_b200.backend.host_ops`` must give exactly what the
reference's own CPU backend gives (src/devproc/backend/cpu/ops.py:24-251) on
the same tokenizer and texts: ``tests/golden/tokenizer_golden.json`` holds
its outputs, recorded by ``tests/golden/make_tokenizer_golden.py`` from the
reference run in this container.  A function that mixes host ops and tensor
ops compiles to a host prologue, one device plan and a host epilogue.
"""

import json
from pathlib import Path

import pytest
import torch

import devproc
from devproc_b200.backend.b200.host_program import HostDeviceProgram
from devproc_b200.backend.host_ops import TokenizerCache, run_host_op, split_host_ops
from devproc_b200.dsl import ops as dsl
from devproc_b200.ir.base import Value
from devproc_b200.ir.ops import OpBuilder
from devproc_b200.ir.types import StringType, TensorType

GOLDEN = Path(__file__).resolve().parent / "golden"
TOK = str(GOLDEN / "tokenizer")


@pytest.fixture(scope="module")
def golden():
    return json.loads((GOLDEN / "tokenizer_golden.json").read_text())


def _run(op, env, cache):
    run_host_op(op, env, cache)
    return env[op.outputs[0].name]


def test_tokenizer_handlers_match_reference(golden):
    cache = TokenizerCache()
    env = {}
    load = OpBuilder.load_tokenizer(TOK)
    _run(load, env, cache)
    for i, text in enumerate(golden["texts"]):
        txt = Value(f"t{i}", StringType())
        env[txt.name] = text
        enc = OpBuilder.tokenize_encode(load.outputs[0], txt)
        ids = _run(enc, env, cache)
        assert ids.dtype == torch.int32 and ids.shape == (2048,)
        assert ids.tolist() == golden["encode"][i], f"text {i}"
        dec = OpBuilder.tokenize_decode(load.outputs[0], enc.outputs[0])
        assert _run(dec, env, cache) == golden["decode"][i]
        assert int(_run(OpBuilder.string_length(txt), env, cache)) == golden["length"][i]


def test_string_and_dict_handlers_match_reference(golden):
    cache = TokenizerCache()
    a, b = Value("a", StringType()), Value("b", StringType())
    env = {"a": golden["texts"][0], "b": golden["texts"][1]}
    assert _run(OpBuilder.string_concat(a, b), env, cache) == golden["concat"]
    assert _run(OpBuilder.string_slice(b, 7, 20), env, cache) == golden["slice"]
    assert _run(OpBuilder.string_format(a), env, cache) == golden["format"]
    d = OpBuilder.dict_create(StringType(), TensorType((3,), "float32", "cpu"))
    _run(d, env, cache)
    v = Value("v", TensorType((3,), "float32", "cpu"))
    env["v"] = torch.tensor([1.0, 2.0, 3.0])
    s = OpBuilder.dict_set(d.outputs[0], a, v)
    _run(s, env, cache)
    s2 = OpBuilder.dict_set(s.outputs[0], b, v)
    _run(s2, env, cache)
    assert _run(OpBuilder.dict_get(s2.outputs[0], a), env, cache).tolist() == golden["dict_get"]
    assert int(_run(OpBuilder.dict_size(s2.outputs[0]), env, cache)) == golden["dict_size"]
    with pytest.raises(KeyError):
        _run(OpBuilder.dict_get(s2.outputs[0], Value("c", StringType())), dict(env, c="missing"), cache)


@devproc.kernel
def tagger(text, emb, w, b):
    """Text -> token ids (host) -> embedding -> linear -> argmax (device) -> text (host)."""
    tok = dsl.load_tokenizer(TOK)
    ids = dsl.tokenize_encode(tok, text)
    x = dsl.embedding(ids, emb)
    pred = dsl.argmax(dsl.linear(x, w, b), dtype="int32")
    return dsl.tokenize_decode(tok, pred)


def _weights(vocab=64, dim=32, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(vocab, dim, generator=g), torch.randn(vocab, dim, generator=g) * 0.5,
            torch.zeros(vocab))


def test_mixed_program_splits_into_host_device_host():
    emb, w, b = _weights()
    fn = devproc.parse_ir(tagger, "example", emb, w, b)
    prologue, sub, epilogue, dev_in, dev_out = split_host_ops(fn)
    assert [o.name for o in prologue] == ["load_tokenizer", "tokenize_encode"]
    assert [o.name for o in sub.block.ops] == ["embedding", "linear", "argmax"]
    assert [o.name for o in epilogue] == ["tokenize_decode"]
    assert dev_in[0] == prologue[1].outputs[0].name and set(dev_in[1:]) == {"emb", "w", "b"}
    prog = devproc.compile(tagger, "example", emb, w, b)
    assert isinstance(prog, HostDeviceProgram)
    assert prog.input_names == ["text", "emb", "w", "b"] and len(prog.device.spec.records) >= 2


def test_mixed_program_save_load_keeps_host_steps(tmp_path):
    emb, w, b = _weights()
    prog = devproc.compile(tagger, "example", emb, w, b)
    devproc.save(prog, str(tmp_path / "tagger"))
    back = devproc.load(str(tmp_path / "tagger"))
    assert isinstance(back, HostDeviceProgram)
    assert back.host_meta() == prog.host_meta()
    assert back.device.spec.plan == prog.device.spec.plan
