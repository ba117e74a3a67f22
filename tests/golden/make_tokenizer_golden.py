"""Tokenizer fixture and golden vectors from the reference's own CPU handlers.

There is no network and no tokenizer checkpoint in this image, so the fixture
is a small word-level tokenizer built here with the ``tokenizers`` library and
saved with ``transformers`` as ``tests/golden/tokenizer/`` (a [PAD] token at
id 0, [UNK] at id 1, 62 lowercase words).  The golden vectors are what the
reference's CPU backend computes with it: its ``handle_tokenize_encode`` and
``handle_tokenize_decode`` (src/devproc/backend/cpu/ops.py:38-86) and its
string and dict handlers (:91-218), run through its own
``CPULoweringContext`` (backend/cpu/codegen.py:20-71) on reference IR ops.
They are written to ``tests/golden/tokenizer_golden.json``.

Usage (in a container that has the reference tree):
    python tests/golden/make_tokenizer_golden.py --ref-src <DevProc checkout>/src
or with DEVPROC_REF_SRC set to that folder.
"""

import argparse
import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
TOK_DIR = HERE / "tokenizer"

WORDS = ("the a an robot arm picks places moves lifts holds drops opens closes pushes pulls turns red green blue "
         "yellow black white small large cup block box bowl plate bottle door drawer lid cloth sponge spoon fork "
         "knife towel on in under over near left right top bottom front back table shelf sink counter floor "
         "please then and slowly carefully now").split()
TEXTS = ["the robot arm picks the red cup",
         "please place the small blue block in the bowl then close the drawer",
         "pick up the zebra",  # an out-of-vocabulary word -> [UNK]
         "",
         " ".join(["move the box left"] * 700)]  # longer than 2048 tokens: truncated


def build_fixture() -> None:
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab = {"[PAD]": 0, "[UNK]": 1}
    for w in WORDS:
        vocab.setdefault(w, len(vocab))
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, pad_token="[PAD]", unk_token="[UNK]")
    TOK_DIR.mkdir(exist_ok=True)
    fast.save_pretrained(str(TOK_DIR))


CHILD = r'''
import json, sys
sys.path.insert(0, REF_SRC)
import torch
from devproc.ir.base import Value
from devproc.ir.types import StringType, TensorType
from devproc.ir.ops import OpBuilder
from devproc.backend.cpu.codegen import CPULoweringContext
from devproc.backend.cpu import ops as cpu_ops
tok_dir, texts = sys.argv[1], json.loads(sys.argv[2])
ctx = CPULoweringContext()
load = OpBuilder.load_tokenizer(tok_dir)
cpu_ops.handle_op(load, ctx)
res = {"encode": [], "decode": [], "length": [], "concat": None, "slice": None, "format": None, "dict_size": None}
for i, t in enumerate(texts):
    txt = Value(f"text{i}", StringType())
    ctx.set_string(txt.name, t)
    enc = OpBuilder.tokenize_encode(load.outputs[0], txt)
    cpu_ops.handle_op(enc, ctx)
    ids = ctx.get_tensor(enc.outputs[0].name)
    res["encode"].append(ids.tolist())
    dec = OpBuilder.tokenize_decode(load.outputs[0], enc.outputs[0])
    cpu_ops.handle_op(dec, ctx)
    res["decode"].append(ctx.get_string(dec.outputs[0].name))
    ln = OpBuilder.string_length(txt)
    cpu_ops.handle_op(ln, ctx)
    res["length"].append(int(ctx.get_tensor(ln.outputs[0].name)))
a, b = Value("a", StringType()), Value("b", StringType())
ctx.set_string("a", texts[0]); ctx.set_string("b", texts[1])
op = OpBuilder.string_concat(a, b); cpu_ops.handle_op(op, ctx); res["concat"] = ctx.get_string(op.outputs[0].name)
op = OpBuilder.string_slice(b, 7, 20); cpu_ops.handle_op(op, ctx); res["slice"] = ctx.get_string(op.outputs[0].name)
op = OpBuilder.string_format(a); cpu_ops.handle_op(op, ctx); res["format"] = ctx.get_string(op.outputs[0].name)
d = OpBuilder.dict_create(StringType(), TensorType((3,), "float32", "cpu")); cpu_ops.handle_op(d, ctx)
v = Value("v", TensorType((3,), "float32", "cpu")); ctx.set_tensor("v", torch.tensor([1.0, 2.0, 3.0]))
s = OpBuilder.dict_set(d.outputs[0], a, v); cpu_ops.handle_op(s, ctx)
s2 = OpBuilder.dict_set(s.outputs[0], b, v); cpu_ops.handle_op(s2, ctx)
g = OpBuilder.dict_get(s2.outputs[0], a); cpu_ops.handle_op(g, ctx)
n = OpBuilder.dict_size(s2.outputs[0]); cpu_ops.handle_op(n, ctx)
res["dict_get"] = ctx.get_tensor(g.outputs[0].name).tolist()
res["dict_size"] = int(ctx.get_tensor(n.outputs[0].name))
print(json.dumps(res))
'''


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default=os.environ.get("DEVPROC_REF_SRC"),
                    help="the reference's src folder (default: $DEVPROC_REF_SRC)")
    ref_src = ap.parse_args().ref_src
    if not ref_src or not (Path(ref_src) / "devproc").is_dir():
        raise SystemExit("give the reference's src folder with --ref-src or DEVPROC_REF_SRC")
    build_fixture()
    code = CHILD.replace("REF_SRC", repr(ref_src))
    r = subprocess.run([sys.executable, "-c", code, str(TOK_DIR), json.dumps(TEXTS)], capture_output=True,
                       text=True, timeout=600)
    if r.returncode != 0:
        raise SystemExit(r.stderr)
    res = json.loads(r.stdout.strip().splitlines()[-1])
    res["texts"] = TEXTS
    (HERE / "tokenizer_golden.json").write_text(json.dumps(res) + "\n")
    print("encoded lengths:", [len(e) for e in res["encode"]], "first ids:", res["encode"][0][:10])


if __name__ == "__main__":
    main()
