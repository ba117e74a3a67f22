"""pi0.5-shaped policy (scaled down) through the FX frontend on the GPU,
against the CPU oracle and torch eager; plus the ops it adds (slice, cat,
expand, rope, grouped-query attention over key counts that are not a
multiple of 8).  bf16 bar: |Δ| ≤ 2e-2 · (max|ref| + |ref|)."""

import pytest
import torch

import devproc
from devproc_b200 import workloads
from devproc_b200.ir.function import Function
from devproc_b200.ir.ops import OpBuilder
from devproc_b200.ir.types import TensorType
from oracle import interp

pytestmark = pytest.mark.gpu


def small_policy():
    return workloads.Pi05Policy(cams=2, text=8, vocab=1000, width=128, layers=2, heads=4, kv_heads=1, head_dim=32,
                                mlp=256, expert_width=64, expert_layers=2, expert_mlp=128, horizon=10,
                                action_dim=8, steps=3, vit=dict(layers=1, dim=64, heads=2, mlp=128, image=56)).eval()


def _close(got, ref, tol=2e-2):
    got, ref = got.float(), ref.float()
    bound = tol * (ref.abs().max() + ref.abs())
    assert ((got - ref).abs() <= bound).all(), (got - ref).abs().max()


def test_small_policy_matches_oracle_and_eager(cuda):
    m = small_policy()
    g = torch.Generator().manual_seed(3)
    pix = torch.randn(4, 3, 56, 56, generator=g).bfloat16()
    ids = torch.randint(0, 1000, (2, 8), generator=g, dtype=torch.int32)
    noise = torch.randn(2, 10, 8, generator=g)
    prog = devproc.compile(m, pix, ids, noise)
    ir = prog.ir_function
    names = {"l_pixels_": pix, "l_text_ids_": ids, "l_noise_": noise}
    inputs = {v.name: names[v.name] for v in ir.inputs if v.name not in ir.constants}
    got = prog.run(**inputs)[0]
    ref = interp.run_function(ir, inputs)[0]
    _close(got, ref)
    with torch.no_grad():
        eager = m(pix, ids, noise)
    _close(got, eager, 5e-2)


def _fn(build, *examples):
    fn = Function("t")
    vals = []
    for i, t in enumerate(examples):
        v = OpBuilder.input(f"x{i}", TensorType(tuple(t.shape), str(t.dtype).replace("torch.", ""))).outputs[0]
        fn.add_input(v)
        vals.append(v)
    ops = build(*vals)
    for op in ops:
        fn.add_op(op)
    fn.output = ops[-1].outputs[0]
    return fn


def _run(fn, *xs):
    from devproc_b200.backend.b200 import B200Compiler
    prog = B200Compiler().compile(fn)
    feed = {f"x{i}": x for i, x in enumerate(xs)}
    return prog.run(**feed)[0], interp.run_function(fn, feed)[0]


@pytest.mark.parametrize("half_tables", [False, True])
def test_rope_program(cuda, half_tables):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 3, 20, 64, generator=g).bfloat16()
    from devproc_b200.torch_ops import rope_tables
    c, s = rope_tables(20, 64)
    if half_tables:
        c, s = c[:, :32].contiguous(), s[:, :32].contiguous()
    got, ref = _run(_fn(lambda a, b, d: [OpBuilder.rope(a, b, d)], x, c, s), x, c, s)
    _close(got, ref)


@pytest.mark.parametrize("xdt,tdt,half,bcast", [
    (torch.bfloat16, torch.bfloat16, False, False),
    (torch.bfloat16, torch.float32, True, False),
    (torch.float16, torch.float16, False, True),
    (torch.float32, torch.bfloat16, False, False),
    (torch.float32, torch.float32, True, True),
])
def test_rope_kernel_bit_exact(cuda, xdt, tdt, half, bcast):
    """``dp_rope`` through the C ABI on a token-major column block of a fused
    projection (x[b, h, r] at b·R·W + r·W + off + h·D), against the torch-level
    op on the CPU: the same fp32 products and sums, so the bits agree."""
    from devproc_b200 import _native as N
    from devproc_b200.torch_ops import rope, rope_tables
    B, H, R, D, W, off = 3, 4, 37, 64, 7 * 64, 64
    g = torch.Generator().manual_seed(5)
    proj = torch.randn(B, R, W, generator=g).to(xdt)
    x = proj[:, :, off:off + H * D].view(B, R, H, D).transpose(1, 2)  # [B, H, R, D], strided
    c, s_ = rope_tables(R, D)
    if half:
        c, s_ = c[:, :D // 2].contiguous(), s_[:, :D // 2].contiguous()
    c, s_ = c.to(tdt), s_.to(tdt)
    if bcast:  # a per-sample table, broadcast over heads
        c = torch.stack([c.roll(i, 0) for i in range(B)])[:, None]
        s_ = torch.stack([s_.roll(i, 0) for i in range(B)])[:, None]
    ref = rope(x, c, s_)
    dproj, dc, ds = proj.to(cuda), c.to(cuda).contiguous(), s_.to(cuda).contiguous()
    out = torch.empty(B, H, R, D, dtype=xdt, device=cuda)
    es = proj.element_size()
    p = N.RopeParams()
    p.batch, p.heads, p.rows, p.dim = B, H, R, D
    p.x_sb, p.x_sh, p.x_sr = R * W, D, W
    p.o_sb, p.o_sh, p.o_sr = H * R * D, R * D, D
    cols = c.shape[-1]
    p.t_sb, p.t_sh, p.t_sr = (R * cols if bcast else 0), 0, cols
    p.half_table = int(half)
    p.x_dtype = N.DTYPE_CODE[str(xdt).replace("torch.", "")]
    p.t_dtype = N.DTYPE_CODE[str(tdt).replace("torch.", "")]
    N.rope(p, dproj.data_ptr() + off * es, dc, ds, out)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), ref)


def test_slice_cat_expand_regions(cuda):
    g = torch.Generator().manual_seed(2)
    x = torch.randn(3, 40, 24, generator=g)
    y = torch.randn(3, 8, 24, generator=g)
    z = torch.randn(1, 1, 24, generator=g)

    def build(a, b, c):
        s1 = OpBuilder.slice(a, 1, 5, 37, 2)          # [3, 16, 24] strided, offset
        s2 = OpBuilder.slice(a, 2, 8, 24)             # [3, 40, 16] offset 8
        ct = OpBuilder.cat([s1.outputs[0], b], 1)     # [3, 24, 24]
        ex = OpBuilder.expand(c, (3, 24, 24))
        ad = OpBuilder.add(ct.outputs[0], ex.outputs[0])
        s3 = OpBuilder.slice(s2.outputs[0], 1, 0, 24)  # [3, 24, 16]
        s4 = OpBuilder.slice(ad.outputs[0], 2, 4, 20)  # [3, 24, 16]
        out = OpBuilder.binary("mul", s3.outputs[0], s4.outputs[0])
        return [s1, s2, ct, ex, ad, s3, s4, out]

    got, ref = _run(_fn(build, x, y, z), x, y, z)
    assert torch.allclose(got, ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("S", [50, 300, 866])
def test_gqa_attention_odd_key_counts(cuda, S):
    """8 query heads over 1 key/value head, key counts not a multiple of 8
    (padded score rows), fused and separate softmax paths."""
    g = torch.Generator().manual_seed(S)
    q = torch.randn(2, 8, 24, 64, generator=g).bfloat16()
    k = torch.randn(2, 1, S, 64, generator=g).bfloat16()
    v = torch.randn(2, 1, S, 64, generator=g).bfloat16()
    got, ref = _run(_fn(lambda a, b, c: [OpBuilder.sdpa(a, b, c)], q, k, v), q, k, v)
    _close(got, ref)
