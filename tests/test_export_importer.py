"""torch.export importer: ExportedProgram → IR → oracle / lowering.

The reference plans ``torch.export`` as the model entry point (CLAUDE.md:9,
docs/MVP实施计划.md:146-185) with parameters as IR constants; these tests
check that an exported module gives the same IR semantics (oracle against
eager) and the same launch plan as the Dynamo frontend.
"""

import re

import pytest
import torch

import devproc_b200 as devproc
from devproc_b200 import workloads
from oracle import interp


def _run_ir(fn, *inputs):
    names = [v.name for v in fn.inputs if v.name not in fn.constants]
    return interp.run_function(fn, dict(zip(names, inputs)))


def _labels(prog):
    """Record labels with SSA value numbers (which differ between frontends) masked."""
    return [re.sub(r"%v\d+", "%v", r["label"]) for r in prog.spec.records]


def test_token_pipeline_export_matches_eager():
    m = workloads.TokenPipeline().eval()
    ids = workloads.token_ids()
    ep = torch.export.export(m, (ids,))
    fn = devproc.from_export(ep, backend="ir")
    assert [v.name for v in fn.inputs if v.name not in fn.constants] == ["ids"]
    assert len(fn.constants) == 9  # emb, fc1 w/b, fc2 w/b, ln w/b, head w/b
    assert [op.name for op in fn.block.ops] == ["embedding", "linear", "gelu", "linear", "layer_norm", "linear",
                                               "argmax", "to"]
    got = _run_ir(fn, ids)[0]
    ref = m(ids)
    assert got.dtype == torch.int32 and torch.equal(got, ref)


def test_token_pipeline_export_plan_equals_dynamo_plan():
    m = workloads.TokenPipeline().eval()
    ids = workloads.token_ids()
    a = devproc.compile(m, ids)
    b = devproc.compile(m, ids, method="export")
    assert _labels(a) == _labels(b)
    assert a.spec.arena_bytes == b.spec.arena_bytes


def test_vit_export_matches_eager_and_dynamo_plan():
    m = workloads.VitClassifier(layers=1, dim=128, heads=4, mlp=256, classes=16, image=56,
                                dtype=torch.float32, logits=True).eval()
    x = torch.randn(2, 3, 56, 56)
    fn = devproc.from_torch(m, x, backend="ir", method="export")
    got = _run_ir(fn, x)[0]
    ref = m(x)
    assert torch.allclose(got, ref, rtol=1e-4, atol=1e-5)
    mb = workloads.VitClassifier(layers=1, dim=128, heads=4, mlp=256, classes=16).eval()
    xb = torch.randn(2, 3, 224, 224).bfloat16()
    assert _labels(devproc.compile(mb, xb)) == _labels(devproc.compile(mb, xb, method="export"))


def test_small_policy_export_plan_equals_dynamo_plan():
    """The policy's buffers (rotary tables, time embedding) arrive as lifted
    buffers, its ``t_emb[s]`` / ``cos[:n]`` as select / slice overloads."""
    m = workloads.Pi05Policy(cams=2, text=8, vocab=1000, width=128, layers=2, heads=4, kv_heads=1, head_dim=32,
                             mlp=256, expert_width=64, expert_layers=2, expert_mlp=128, horizon=10, action_dim=8,
                             steps=3, vit=dict(layers=1, dim=64, heads=2, mlp=128, image=56)).eval()
    args = (torch.randn(4, 3, 56, 56).bfloat16(), torch.randint(0, 1000, (2, 8), dtype=torch.int32),
            torch.randn(2, 10, 8))
    ep = devproc.ir.export_importer.export_module(m, *args)
    assert _labels(devproc.compile(m, *args)) == _labels(devproc.compile(ep))


def test_small_policy_export_oracle_matches_eager():
    m = workloads.Pi05Policy(cams=1, text=4, vocab=100, width=64, layers=1, heads=2, kv_heads=1, head_dim=16,
                             mlp=128, expert_width=32, expert_layers=1, expert_mlp=64, horizon=4, action_dim=8,
                             steps=2, vit=dict(layers=1, dim=32, heads=2, mlp=64, image=28),
                             dtype=torch.float32).eval()
    args = (torch.randn(1, 3, 28, 28), torch.randint(0, 100, (1, 4), dtype=torch.int32), torch.randn(1, 4, 8))
    fn = devproc.from_torch(m, *args, backend="ir", method="export")
    got = _run_ir(fn, *args)[0]
    with torch.no_grad():
        ref = m(*args)
    assert torch.allclose(got, ref, rtol=1e-4, atol=1e-5)


def test_aten_only_forms():
    """select.int, slice.Tensor with open ends, upsample_bilinear2d, eval-mode
    dropout and a float cast, against eager on the oracle."""

    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.drop = torch.nn.Dropout(0.5)
            self.register_buffer("scale", torch.tensor([0.5, 2.0, -1.0]))

        def forward(self, img, x):
            r = torch.nn.functional.interpolate(img.float(), size=(7, 9), mode="bilinear", align_corners=False)
            y = self.drop(x[:, 1]) * 3.0
            z = x[1:, :, -4:] - x[:1, :, :4]
            return r * self.scale[:, None, None], y, z.sum(-1)

    m = M().eval()
    img = torch.randint(0, 256, (2, 3, 16, 20), dtype=torch.uint8)
    x = torch.randn(3, 5, 8)
    fn = devproc.from_torch(m, img, x, backend="ir", method="export")
    got = _run_ir(fn, img, x)
    ref = m(img, x)
    assert len(got) == 3
    for g_, r_ in zip(got, ref):
        assert g_.shape == r_.shape and torch.allclose(g_, r_, rtol=1e-5, atol=1e-4)


def test_state_mutation_is_rejected():
    class Counter(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.register_buffer("n", torch.zeros(1))

        def forward(self, x):
            self.n.add_(1)
            return x + self.n

    ep = torch.export.export(Counter(), (torch.randn(4),))
    with pytest.raises(ValueError, match="mutates state"):
        devproc.from_export(ep, backend="ir")


def test_decomposed_core_aten_token_pipeline():
    """``ep.run_decompositions()`` (core ATen: addmm over a transposed weight,
    native_layer_norm with its tuple result, permute, _to_copy) imports to the
    same plan as the high-level export, and the oracle matches eager."""
    m = workloads.TokenPipeline().eval()
    ids = workloads.token_ids()
    ep = torch.export.export(m, (ids,))
    dec = ep.run_decompositions()
    fn = devproc.from_export(dec, backend="ir")
    assert "linear" in [op.name for op in fn.block.ops]
    assert torch.equal(_run_ir(fn, ids)[0], m(ids))
    assert _labels(devproc.compile(ep)) == _labels(devproc.compile(dec))


def test_decomposed_core_aten_patchify_softmax():
    """convolution (patchify), _softmax, addmm without a transposed weight."""

    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.patch = torch.nn.Conv2d(3, 16, kernel_size=4, stride=4)
            self.w = torch.nn.Parameter(torch.randn(16, 5))
            self.b = torch.nn.Parameter(torch.randn(5))

        def forward(self, x):
            y = self.patch(x).flatten(2).transpose(1, 2)       # [B, 16 patches, 16]
            z = torch.addmm(self.b, y.reshape(-1, 16), self.w)  # weight used as [K, N]
            return torch.softmax(z, -1)

    m = M().eval()
    x = torch.randn(2, 3, 16, 16)
    ep = torch.export.export(m, (x,)).run_decompositions()
    fn = devproc.from_export(ep, backend="ir")
    got = _run_ir(fn, x)[0]
    with torch.no_grad():
        ref = m(x)
    assert torch.allclose(got, ref, rtol=1e-4, atol=1e-5)


def test_aten_softmax_half_to_float_gives_fp32():
    """aten._softmax(x, dim, half_to_float=True) on bf16 x returns fp32."""

    class M(torch.nn.Module):
        def forward(self, x):
            return torch.ops.aten._softmax(x, -1, True)

    x = torch.randn(4, 40).bfloat16()
    ep = torch.export.export(M(), (x,))
    fn = devproc.from_export(ep, backend="ir")
    assert [op.name for op in fn.block.ops] == ["to", "softmax"]
    got = _run_ir(fn, x)[0]
    assert got.dtype == torch.float32
    assert torch.allclose(got, torch.softmax(x.float(), -1), rtol=1e-5, atol=1e-7)
