"""Batch separability and chunked programs (host-transfer streaming).

A program whose samples are independent can run on chunks of its batch while
the transfers of neighbouring chunks overlap.  These tests pin the analysis
(which programs qualify) and that the chunk program computes exactly the
full program's rows, on the oracle."""

import pytest
import torch

import devproc_b200 as devproc
from devproc_b200 import workloads
from devproc_b200.backend.b200.rebatch import batch_factors, rebatch
from oracle import interp


def _ir(m, *x):
    return devproc.from_torch(m, *x, backend="ir")


def _runtime_names(fn):
    return [v.name for v in fn.inputs if v.name not in (getattr(fn, "constants", None) or {})]


def _check_chunk_matches(fn, inputs, b):
    """Oracle of the b-sample program on every chunk == rows of the full run."""
    names = _runtime_names(fn)
    full = interp.run_function(fn, dict(zip(names, inputs)))
    sub = rebatch(fn, b)
    B = inputs[0].shape[0]
    for lo in range(0, B, b):
        part = interp.run_function(sub, {n: x[lo:lo + b] for n, x in zip(names, inputs)})
        for f_, p_ in zip(full, part):
            rows = f_.shape[0] // B
            assert torch.equal(f_[lo * rows:(lo + b) * rows], p_), (f_.shape, p_.shape)


def test_preprocess_is_separable_and_streams():
    imgs = workloads.preprocess_images(4)
    fn = devproc.parse_ir(workloads.vision_preprocess, imgs)
    B, fac, why = batch_factors(fn)
    assert B == 4 and why == ""
    _check_chunk_matches(fn, [imgs], 2)
    big = torch.zeros(64, 480, 640, 3, dtype=torch.uint8)
    prog = devproc.compile(workloads.vision_preprocess, big)
    assert prog.stream_chunk == 8 and 64 % prog.stream_chunk == 0
    assert prog._chunk.spec.inputs[0].shape == [8, 480, 640, 3]
    assert prog._chunk.spec.outputs[0].shape == [8, 3, 224, 224]


def test_token_pipeline_is_separable_but_not_streamed():
    """Rows of [B·L, D] after the flattening reshape belong to samples in
    order, so the pipeline is separable; with GEMMs it is compute-bound and
    keeps one whole-batch run."""
    m = workloads.TokenPipeline()
    ids = workloads.token_ids()
    fn = _ir(m, ids)
    B, fac, _ = batch_factors(fn)
    assert B == 8
    _check_chunk_matches(fn, [ids], 2)
    assert devproc.compile(m, ids).stream_chunk is None


def test_vit_is_separable():
    m = workloads.VitClassifier(layers=1, dim=64, heads=2, mlp=128, classes=10, image=28,
                                dtype=torch.float32).eval()
    x = torch.randn(4, 3, 28, 28)
    fn = _ir(m, x)
    assert batch_factors(fn)[0] == 4
    _check_chunk_matches(fn, [x], 2)


@pytest.mark.parametrize("body", [
    lambda x: x.sum(0),                       # reduction along the batch dim
    lambda x: x.reshape(1, -1) * 2.0,         # merges samples into one row
    lambda x: torch.cat([x, x], 0),           # cat along the batch dim
    lambda x: torch.softmax(x, 0),            # normalises across samples
    lambda x: x @ x.transpose(0, 1),          # contracts over samples
    lambda x: x - x.mean(0, keepdim=True),    # broadcasts a cross-sample value
])
def test_cross_sample_programs_are_not_separable(body):
    class M(torch.nn.Module):
        def forward(self, x):
            return body(x)

    fn = _ir(M(), torch.randn(4, 6))
    B, _, why = batch_factors(fn)
    assert B is None and why


def test_shared_constants_broadcast_over_samples():
    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Linear(6, 5)
            self.bias = torch.nn.Parameter(torch.randn(5))

        def forward(self, x):
            y = self.lin(x) + self.bias
            return torch.softmax(y, -1), y.reshape(-1).argmax(-1, keepdim=True) * 0 + y[:, :1].argmax(-1)

    m = M()
    x = torch.randn(6, 6)
    fn = _ir(m, x)
    B, fac, why = batch_factors(fn)
    # the second output reduces the flattened batch: not separable
    assert B is None and "argmax" in why

    class N1(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Linear(6, 5)
            self.bias = torch.nn.Parameter(torch.randn(5))

        def forward(self, x):
            return torch.softmax(self.lin(x) + self.bias, -1)

    fn = _ir(N1(), x)
    assert batch_factors(fn)[0] == 6
    _check_chunk_matches(fn, [x], 3)


def test_chunk_program_survives_save_and_load(tmp_path):
    big = torch.zeros(32, 480, 640, 3, dtype=torch.uint8)
    prog = devproc.compile(workloads.vision_preprocess, big)
    assert prog.stream_chunk is not None
    devproc.save(prog, str(tmp_path / "pre"))
    again = devproc.load(str(tmp_path / "pre"))
    assert again.stream_chunk == prog.stream_chunk
    assert again._chunk.spec.plan == prog._chunk.spec.plan
    assert again.spec.plan == prog.spec.plan
