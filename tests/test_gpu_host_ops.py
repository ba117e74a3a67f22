"""A tokenizer -> embedding -> linear -> argmax -> decode program end to end.

The host prologue encodes the text with the reference's tokenizer semantics
(checked bit-exact against the reference's own handler output in
``tests/golden/tokenizer_golden.json``), the GPU plan gathers embeddings and
runs the linear and the argmax, and the host epilogue decodes the predicted
ids.  The device ids must equal the CPU oracle's wherever the top-2 logit gap
exceeds 1e-4 of the largest logit (fp32 bar), and the returned text must be
the decoding of the device ids.
"""

import json
from pathlib import Path

import pytest
import torch

import devproc
from devproc_b200.backend.host_ops import TokenizerCache
from oracle import interp

from test_host_ops import TOK, _weights, tagger

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_tokenizer_program_end_to_end(cuda):
    golden = json.loads((GOLDEN / "tokenizer_golden.json").read_text())
    emb, w, b = _weights()
    prog = devproc.compile(tagger, "example", emb, w, b)
    enc_name = prog.device_inputs[0]
    tok = TokenizerCache().get(TOK)
    for i in (0, 1, 4):
        text = golden["texts"][i]
        got_text = prog.run(text=text, emb=emb, w=w, b=b)[0]
        ids = torch.tensor(golden["encode"][i], dtype=torch.int32)
        feed = {enc_name: ids, "emb": emb, "w": w, "b": b}
        dev_ids = prog.device.run(**{n: feed[n] for n in prog.device.input_names})[0]
        sub = prog.device.ir_function
        ref_ids = interp.run_function(sub, feed)[0]
        logits = (emb[ids.long()] @ w.T + b)
        top2 = logits.topk(2, -1).values
        decided = (top2[:, 0] - top2[:, 1]) > 1e-4 * logits.abs().max()
        assert decided.float().mean() > 0.99
        assert torch.equal(dev_ids[decided], ref_ids[decided]), f"text {i}"
        want = tok.decode([t for t in dev_ids.tolist() if t != tok.pad_token_id])
        assert got_text == want
