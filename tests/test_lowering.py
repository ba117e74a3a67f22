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
    # each fp32 linear is one 3xTF32 tensor-core GEMM over a [hi | hi | lo] operand that its producer
    # writes directly (the embedding gathers rows of a table split at compile time, the fc1 split-K
    # reduce and the LayerNorm store the three blocks); the two M = 1024 linears with few output tiles
    # split K (a batched GEMM plus a reduce that applies the epilogue); the head's argmax (and the int32
    # cast) is reduced in the head GEMM's epilogue between a clear and a conversion of one key per row,
    # so the 1024 x 32000 logits are never stored
    assert kernels(prog) == ["embedding", "gemm", "splitk", "gemm", "splitk", "rowreduce",
                             "argmax_keys", "gemm", "argmax_keys"]
    assert all("3xtf32" in lb for lb in labels if lb.startswith("gemm"))
    assert "splitk2" in labels[1] and "splitk8" in labels[3] and "splitk" not in labels[7]
    assert f"epi{N.DP_EPI_BIAS | N.DP_EPI_GELU_ERF}" in labels[2] and "3xtf32 operand" in labels[2]
    assert "3xtf32 operand" not in labels[4] and "3xtf32 operand" in labels[5]
    assert labels[0] == "embedding 1024x1536"
    assert "argmax" in labels[7] and f"epi{N.DP_EPI_BIAS | N.DP_EPI_ARGMAX}" in labels[7]
    assert "int32" in labels[8]
    assert prog.spec.arena_bytes < 64 << 20
    w3 = [c for c in prog.spec.consts if c.name.endswith("|3xtf32")]
    assert len(w3) == 3 and w3[0].shape[1] == 3 * 512
    assert prog.spec.outputs[0].dtype == "int32"
    # constants are bound once; one runtime input
    assert [i.name for i in prog.spec.inputs] == ["l_ids_"]


def test_ragged_last_wave_gemm_splits_by_k_stage():
    """With stream-K switched on, a bf16 linear with fewer 256 x 256 tiles than
    CTA pairs (3,200 x 1,024, K 4,096: 52 tiles for 74 pairs) lowers to one
    stream-K GEMM record with an arena workspace; GEMMs whose last wave is
    full or nearly so, or whose K is short, keep whole tiles."""
    from devproc_b200.backend.b200.lowering import Lowerer, streamk_bytes
    m = torch.nn.Linear(4096, 1024).to(torch.bfloat16)
    x = torch.randn(3200, 4096).to(torch.bfloat16)
    assert kernels(devproc.compile(m, x)) == ["gemm"]  # opt-in: whole tiles by default
    Lowerer.use_streamk = True
    try:
        prog = devproc.compile(m, x)
    finally:
        Lowerer.use_streamk = False
    assert kernels(prog) == ["gemm_sk"]
    assert "streamk" in prog.spec.records[0]["label"]
    assert streamk_bytes(3200, 1024, 4096, 1, False, 0) > 74 * 256 * 1024
    assert streamk_bytes(3200, 1024, 4096, 1, False, N.DP_EPI_SOFTMAX) == 0
    assert streamk_bytes(8192, 8192, 8192, 1, False, 0) == 0        # 1,024 tiles: the ragged wave is a small share
    assert streamk_bytes(3200, 4096, 1024, 1, False, 0) == 0        # 208 tiles, 8 K stages each
    assert streamk_bytes(148 * 128, 256, 4096, 1, False, 0) == 0    # 74 pair tiles: one full wave


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


def _small_vit(**kw):
    return workloads.VitClassifier(layers=1, dim=128, heads=4, mlp=256, classes=16, **kw).eval()


def test_tf32_split_is_exact():
    """hi carries the TF32 grid part (low 13 mantissa bits zero) and hi + lo
    reproduces every fp32 weight exactly."""
    from devproc_b200.backend.b200.lowering import Lowerer
    m = workloads.TokenPipeline()
    ir = devproc.from_torch(m, workloads.token_ids(), backend="ir")
    low = Lowerer(ir, ir.constants.keys(), ir.constants).run()
    name = [n for n in low.extra_consts if n.endswith("|3xtf32")][0]
    w3 = low.extra_consts[name]
    K = w3.shape[1] // 3
    hi, lo, hi2 = w3[:, :K], w3[:, K:2 * K], w3[:, 2 * K:]
    assert torch.equal(hi, hi2)
    assert ((hi.view(torch.int32) & 8191) == 0).all()
    orig = ir.constants[name.split("|")[0]].float()
    assert torch.equal(hi + lo, orig)


def test_vit_block_lowering_fusions():
    """q/k/v run as one GEMM over a concatenated weight, the patchify reshape is
    one padded copy, and the position embedding rides the patch GEMM's epilogue."""
    m = _small_vit()
    x = torch.randn(2, 3, 224, 224).bfloat16()
    prog = devproc.compile(m, x)
    labels = [r["label"] for r in prog.spec.records]
    assert labels[0].startswith("copy") and "K588->592" in labels[0]
    patch = labels[1]
    assert patch.startswith("gemm linear M256 N128 K588 b2")
    assert f"epi{N.DP_EPI_BIAS | N.DP_EPI_RESIDUAL}" in patch
    assert sum("linear x3" in lb for lb in labels) == 1
    assert not any(lb.startswith("region add") for lb in labels)
    # the three projection weights are replaced by their concatenation (bound once)
    names = [c.name for c in prog.spec.consts]
    assert not any(n.endswith("attn_modules_q_parameters_weight_") for n in names)
    fused = [n for n in names if "+" in n and n.endswith("_v_parameters_weight_")]
    assert len(fused) == 1
    w = prog._constants[fused[0]]
    ref = torch.cat([m.blocks[0].attn.q.weight, m.blocks[0].attn.k.weight, m.blocks[0].attn.v.weight])
    assert torch.equal(w, ref)
    # the padded patch weight is a compile-time constant
    assert any(n.endswith("|pad592") for n in names)


def test_sibling_linears_alias_slots_and_arena():
    """Each fused output is a column block of one arena buffer, addressed by a
    sub-range slot 16-byte aligned inside its root."""
    from devproc_b200.backend.b200.lowering import Lowerer
    m = _small_vit()
    x = torch.randn(2, 3, 224, 224).bfloat16()
    ir = devproc.from_torch(m, x, backend="ir")
    low = Lowerer(ir, ir.constants.keys(), ir.constants).run()
    subs = [b for b in low.buffers if b.base is not None]
    assert len(subs) == 2  # k and v blocks (q starts at the root)
    for b in subs:
        assert b.offset == b.root.offset + b.base_off and b.offset % 16 == 0
        assert b.base_off in (128 * 2, 256 * 2)
        assert b.offset + b.nbytes == b.root.offset + b.root.nbytes
    assert low.aliases == []  # arena roots need no host binding


def test_sibling_fusion_skips_epilogue_consumers():
    """Two linears on one input where one feeds an activation stay separate, so
    the activation stays in that GEMM's epilogue."""
    class Two(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.a = torch.nn.Linear(64, 32)
            self.b = torch.nn.Linear(64, 32)

        def forward(self, x):
            return torch.relu(self.a(x)) * self.b(x)

    prog = devproc.compile(Two(), torch.randn(8, 64))
    labels = [r["label"] for r in prog.spec.records]
    assert sum(lb.startswith("gemm") for lb in labels) == 2
    assert any(f"epi{N.DP_EPI_BIAS | N.DP_EPI_RELU}" in lb for lb in labels)


def test_unfused_lowering_without_constant_values():
    """Without the constants' values (plan-only lowering) nothing is fused that
    would need a new constant."""
    m = _small_vit()
    x = torch.randn(2, 3, 224, 224).bfloat16()
    ir = devproc.from_torch(m, x, backend="ir")
    low = lower(ir, const_names=ir.constants.keys())
    assert not any("linear x3" in lb for lb in low.labels)
    assert low.extra_consts == {}


def test_small_policy_lowering():
    """The scaled-down pi0.5 policy captures and lowers: one rope region per
    rotated tensor, fused q/k/v, grouped-query attention with padded score
    rows, and expert keys / values joined to the prefix ones by cat copies."""
    m = workloads.Pi05Policy(cams=2, text=8, vocab=1000, width=128, layers=2, heads=4, kv_heads=1, head_dim=32,
                             mlp=256, expert_width=64, expert_layers=2, expert_mlp=128, horizon=10, action_dim=8,
                             steps=3, vit=dict(layers=1, dim=64, heads=2, mlp=128, image=56)).eval()
    pix = torch.randn(4, 3, 56, 56).bfloat16()
    ids = torch.randint(0, 1000, (2, 8), dtype=torch.int32)
    noise = torch.randn(2, 10, 8)
    prog = devproc.compile(m, pix, ids, noise)
    labels = [r["label"] for r in prog.spec.records]
    assert sum(lb.startswith("rope") for lb in labels) == 2 * (2 + 3 * 2)
    assert sum("linear x3" in lb for lb in labels) == 1 + 2 + 3 * 2
    # grouped-query attention (4 query heads per key/value head) as fused attention records;
    # the expert's queries see the 40 prefix keys plus their own 10
    assert any(lb.startswith("attention b2 hkv1 g4 L10 S50 D32") for lb in labels)
    assert sum(lb.startswith("attention") for lb in labels) == 1 + 2 + 3 * 2
    # the expert's keys / values: cat(prefix, new) per layer and step; the prefix part is copied at
    # the first step only (later steps reuse the buffer and copy the 10 new rows), plus cat(img, txt)
    cats = [lb for lb in labels if lb.startswith("cat")]
    assert len(cats) == 2 + 2 * 2 * 2 + 2 * 2 * (3 - 1), cats
    assert prog.spec.outputs[0].shape == [2, 10, 8] and prog.spec.outputs[0].dtype == "float32"


def test_cat_reuses_a_dead_buffer_with_the_same_prefix_only():
    """cat(x, y2) may reuse the buffer of an earlier cat(x, y1) and copy only y2,
    but not while the earlier result (or a view of it) is still to be read."""
    from devproc_b200.dsl import ops as dsl_ops

    @devproc.kernel
    def dead(x, y1, y2):
        a = dsl_ops.cat([x, y1], dim=0)
        s = devproc.sigmoid(a)
        b = dsl_ops.cat([x, y2], dim=0)
        return devproc.add(s, b)

    @devproc.kernel
    def live(x, y1, y2):
        a = dsl_ops.cat([x, y1], dim=0)
        b = dsl_ops.cat([x, y2], dim=0)
        return devproc.add(devproc.transpose(a, (1, 0)), devproc.transpose(b, (1, 0)))

    x, y = torch.randn(6, 16), torch.randn(2, 16)
    cats = lambda prog: [r["label"] for r in prog.spec.records if r["label"].startswith("cat")]
    assert len(cats(devproc.compile(dead, x, y, y))) == 3    # x copied once
    assert len(cats(devproc.compile(live, x, y, y))) == 4    # a is read after b: no reuse


def test_fx_slicing_and_joining():
    """Indexing with slices / ints / None / ..., chunk, split, narrow and cat
    through the FX frontend agree with eager on the oracle."""
    from oracle import interp

    class M(torch.nn.Module):
        def forward(self, x):
            a, b = x.chunk(2, dim=-1)
            c = x[..., 1:7:2, None, :4]
            d = torch.narrow(x, 1, 2, 3)
            e, f, _ = torch.split(x, [3, 4, 1], dim=1)
            return torch.cat([a * b, d.sum(-1, keepdim=True).expand(-1, -1, 4)], 1), c, e + f[:, :3]

    x = torch.randn(2, 8, 8)
    ir = devproc.from_torch(M(), x, backend="ir")
    got = interp.run_function(ir, {ir.inputs[0].name: x})
    ref = M()(x)
    for g_, r_ in zip(got, ref):
        assert torch.allclose(g_, r_, atol=1e-5), (g_.shape, r_.shape)


def test_derived_constants_have_one_slot_each():
    """A fused weight that several records read (the action expert's q/k/v in
    every denoise step) is one constant slot, bound once."""
    m = workloads.Pi05Policy(cams=2, text=8, vocab=1000, width=128, layers=2, heads=4, kv_heads=1, head_dim=32,
                             mlp=256, expert_width=64, expert_layers=2, expert_mlp=128, horizon=10, action_dim=8,
                             steps=3, vit=dict(layers=1, dim=64, heads=2, mlp=128, image=56)).eval()
    prog = devproc.compile(m, torch.randn(4, 3, 56, 56).bfloat16(), torch.randint(0, 1000, (2, 8), dtype=torch.int32),
                           torch.randn(2, 10, 8))
    names = [c.name for c in prog.spec.consts]
    assert len(names) == len(set(names))
