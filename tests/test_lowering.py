"""Lowering: fusion decisions, arena planning and plan serialisation (host only)."""

import random

import pytest
import torch

import devproc
from devproc_b200 import _native as N
from devproc_b200 import workloads
from devproc_b200.backend.b200.lowering import Buffer, collapse_dims, lower, plan_arena


def kernels(prog):
    return [r["kernel"] for r in prog.spec.records]


def test_preprocess_pipeline_is_one_launch():
    prog = devproc.compile(workloads.vision_preprocess, workloads.preprocess_images(4))
    assert kernels(prog) == ["preproc"]
    assert prog.spec.arena_bytes == 0
    assert prog.spec.outputs[0].shape == [4, 3, 224, 224] and prog.spec.outputs[0].dtype == "bfloat16"


def test_token_pipeline_fuses_epilogues_and_argmax_cast():
    m = workloads.TokenPipeline()
    prog = devproc.compile(m, workloads.token_ids())
    labels = [r["label"] for r in prog.spec.records]
    assert kernels(prog) == ["embedding", "gemm", "gemm", "rowreduce", "gemm", "rowreduce"]
    assert f"epi{N.DP_EPI_BIAS | N.DP_EPI_GELU_ERF}" in labels[1]
    assert "argmax" in labels[5] and "int32" in labels[5]
    assert prog.spec.outputs[0].dtype == "int32"
    # constants are bound once; one runtime input
    assert [i.name for i in prog.spec.inputs] == ["l_ids_"]


def test_elementwise_chain_is_one_region():
    @devproc.kernel
    def f(x, y):
        a = devproc.relu(x)
        b = devproc.add(a, y)
        return devproc.sigmoid(b)

    prog = devproc.compile(f, torch.randn(64, 32), torch.randn(32))
    assert kernels(prog) == ["region"]


def test_transpose_is_a_view_folded_into_consumer():
    @devproc.kernel
    def f(x):
        return devproc.relu(devproc.transpose(x, (1, 0)))

    prog = devproc.compile(f, torch.randn(16, 8))
    assert kernels(prog) == ["region"]


def test_arena_offsets_never_overlap_while_live():
    rnd = random.Random(0)
    for trial in range(50):
        bufs = []
        for i in range(30):
            first = rnd.randrange(0, 20)
            b = Buffer("arena", "float32", (rnd.randrange(1, 5000),), f"b{i}")
            b.first, b.last = first, first + rnd.randrange(0, 6)
            bufs.append(b)
        top = plan_arena(bufs)
        for a in bufs:
            assert a.offset % 256 == 0 and a.offset + a.nbytes <= top
            for b in bufs:
                if a is b or a.last < b.first or b.last < a.first:
                    continue
                assert a.offset + a.nbytes <= b.offset or b.offset + b.nbytes <= a.offset


def test_arena_reuses_memory_across_a_chain():
    m = workloads.TokenPipeline()
    prog = devproc.compile(m, workloads.token_ids())
    live_sum = 8 * 128 * (512 + 2048 + 512 + 512 + 32000) * 4
    assert prog.spec.arena_bytes < live_sum


def test_collapse_keeps_channel_dim():
    shape, strides, dmap = collapse_dims((4, 5, 6, 3), [(90, 18, 3, 1), (90, 18, 3, 1)], keep={3})
    assert shape == (120, 3) and dmap[3] == 1
    shape, strides, dmap = collapse_dims((4, 5, 6), [(30, 6, 1)], keep=set())
    assert shape == (120,)


def test_plan_blob_layout():
    prog = devproc.compile(workloads.vision_preprocess, workloads.preprocess_images(2))
    plan = prog.spec.plan
    hdr = N.PlanHeader.from_buffer_copy(plan[:ctypes_size(N.PlanHeader)])
    assert hdr.magic == N.DP_PLAN_MAGIC and hdr.n_records == 1 and hdr.n_slots == 2
    assert len(plan) == ctypes_size(N.PlanHeader) + 2 * ctypes_size(N.PlanSlot) + ctypes_size(N.PlanRecord)


def ctypes_size(cls):
    import ctypes
    return ctypes.sizeof(cls)


def test_save_load_roundtrip_on_host(tmp_path):
    m = workloads.TokenPipeline()
    prog = devproc.compile(m, workloads.token_ids())
    devproc.save(prog, str(tmp_path / "tok"))
    back = devproc.load(str(tmp_path / "tok"))
    assert back.spec.plan == prog.spec.plan
    assert [i.name for i in back.spec.inputs] == [i.name for i in prog.spec.inputs]
    for c in prog.spec.consts:
        assert torch.equal(back._constants[c.name], prog._constants[c.name].detach())


def test_run_without_gpu_fails_loudly():
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    prog = devproc.compile(workloads.vision_preprocess, workloads.preprocess_images(1))
    with pytest.raises(devproc.DevProcError, match="no CUDA device"):
        prog.run(images=workloads.preprocess_images(1))


def test_host_ops_are_rejected():
    @devproc.kernel
    def f(x):
        return x

    fn = f(torch.randn(2))
    from devproc_b200.ir.ops import OpBuilder
    op = OpBuilder.load_tokenizer("gpt2")
    fn.add_op(op)
    with pytest.raises(devproc.CompilationError):
        lower(fn)
