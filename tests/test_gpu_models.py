"""Model pipelines through the FX frontend on the GPU, against the CPU oracle.

bf16 results: |Δ| ≤ 2e-2 · max|ref| + 2e-2 · |ref| (the bf16 bar); argmax
outputs must match wherever the oracle's top-2 logit gap exceeds 5e-2 of the
largest logit magnitude.
"""

import pytest
import torch

import devproc
from devproc_b200 import workloads
from oracle import interp

pytestmark = pytest.mark.gpu


def _runtime_input(ir):
    return [v.name for v in ir.inputs if v.name not in ir.constants][0]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_small_vit_logits(cuda, dtype):
    m = workloads.VitClassifier(layers=2, dim=128, heads=4, mlp=256, classes=16, dtype=dtype, logits=True).eval()
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4, 3, 224, 224, generator=g).to(dtype)
    prog = devproc.compile(m, x)
    got = prog.run(x)[0].float()
    ir = devproc.from_torch(m, x, backend="ir")
    ref = interp.run_function(ir, {_runtime_input(ir): x})[0].float()
    scale = ref.abs().max()
    tol = (1e-4 if dtype == torch.float32 else 2e-2) * (scale + ref.abs())
    assert ((got - ref).abs() <= tol).all(), (got - ref).abs().max()


def test_small_vit_argmax_gap_aware(cuda):
    m = workloads.VitClassifier(layers=2, dim=128, heads=4, mlp=256, classes=16).eval()
    ml = workloads.VitClassifier(layers=2, dim=128, heads=4, mlp=256, classes=16, logits=True).eval()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(8, 3, 224, 224, generator=g).bfloat16()
    got = devproc.compile(m, x).run(x)[0]
    ir = devproc.from_torch(ml, x, backend="ir")
    logits = interp.run_function(ir, {_runtime_input(ir): x})[0].float()
    top2 = logits.topk(2, -1).values
    decided = (top2[:, 0] - top2[:, 1]) > 5e-2 * logits.abs().max()
    assert torch.equal(got[decided], logits.argmax(-1)[decided])
