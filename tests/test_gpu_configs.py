"""Parity at the benchmark configurations' own shapes, against the CPU oracle.

* GEMM 8192 x 2048 x 16384 (bf16 in, fp32 accumulate), the second template
  microbenchmark shape, through the C ABI as the benchmark calls it: sampled
  rows against an fp64 product of the same bf16 operands.
* Row reductions over fp32 [65536, 4096], N(0, 1), all five benchmarked kinds
  (sum, max, argmax, softmax, RMSNorm eps 1e-6 with weight 1), compiled and run
  through ``devproc.compile`` -> ``run``: every row against the oracle.
* The ViT classifier pipeline at its configured shape: uint8 480x640 images ->
  preprocessing -> SigLIP-So400m/14-shaped encoder with all 27 layers (width
  1152, 16 heads of 72, MLP 4304, GELU-tanh, LayerNorm) -> mean-pool -> Linear
  1152 -> 1000 -> argmax, on a sub-batch of 4 images.
* The pi0.5-shaped policy at its configured shape, one sample: 3 camera images
  through the same 27-layer encoder, the Gemma-2B-shaped prefill (18 layers,
  width 2048, 8 query heads over 1 key/value head of 256, GeGLU 16384, RMSNorm,
  RoPE) over 816 tokens, and 10 denoise steps of the 18-layer, 1024-wide action
  expert attending to the prefix keys / values.

Tolerances (stated per test): sum |Δ| <= 1e-6 · Σ|x|; max and argmax exact;
softmax rtol 1e-5; RMSNorm rtol 1e-4; GEMM fp32 |Δ| <= 1e-5 · Σ|a·b| (plus
2^-8 · |ref| for a bf16 result); bf16 models |Δ| <= 2e-2 · (max|ref| + |ref|),
and argmax exact wherever the oracle's top-2 logit gap exceeds 2e-2 of the
largest logit magnitude (the bf16 bar).
"""

import pytest
import torch

import devproc
from devproc_b200 import _native as N
from devproc_b200 import workloads
from devproc_b200.backend.b200 import B200Compiler
from devproc_b200.ir.function import Function
from devproc_b200.ir.ops import OpBuilder
from devproc_b200.ir.types import TensorType
from oracle import interp

pytestmark = pytest.mark.gpu


# ------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("c_dtype", [torch.float32, torch.bfloat16])
def test_gemm_8192x2048x16384_sampled_rows(cuda, c_dtype):
    M, Nn, K = 8192, 2048, 16384
    g = torch.Generator(device=cuda).manual_seed(0)
    a = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    b = torch.randn(Nn, K, device=cuda, generator=g).bfloat16()
    c = torch.empty(M, Nn, device=cuda, dtype=c_dtype)
    p = N.GemmParams()
    p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.batch = M, Nn, K, K, K, Nn, 1
    p.a_dtype = p.b_dtype = N.DP_BF16
    p.c_dtype = N.DTYPE_CODE[str(c_dtype).replace("torch.", "")]
    p.b_layout = N.DP_B_NK
    N.gemm(p, a, b, c)
    torch.cuda.synchronize()
    assert N.device_error_pending(0) == N.DP_DEVERR_NONE
    # first and last rows of the matrix and of 256-row pair tiles, plus random rows
    rows = torch.cat([torch.tensor([0, 127, 128, 255, 256, M - 129, M - 1]),
                      torch.randint(0, M, (57,), generator=torch.Generator().manual_seed(1))]).unique()
    a64 = a[rows.to(cuda)].cpu().double()
    b64 = b.cpu().double()
    ref = a64 @ b64.T
    mag = a64.abs() @ b64.abs().T
    got = c[rows.to(cuda)].cpu().double()
    bound = 1e-5 * mag + (2.0 ** -8 * ref.abs() if c_dtype == torch.bfloat16 else 0.0)
    assert ((got - ref).abs() <= bound).all(), ((got - ref).abs() / mag).max()


# ------------------------------------------------------------- reductions
def _row_fn(kind, rows, cols):
    fn = Function(f"c3b_{kind}")
    x = OpBuilder.input("x", TensorType((rows, cols), "float32")).outputs[0]
    fn.add_input(x)
    if kind == "rms_norm":
        w = OpBuilder.input("w", TensorType((cols,), "float32")).outputs[0]
        fn.add_input(w)
        op = OpBuilder.rms_norm(x, w, eps=1e-6)
    elif kind == "softmax":
        op = OpBuilder.softmax(x, -1)
    elif kind == "argmax":
        op = OpBuilder.argmax(x, -1, dtype="int64")
    else:
        op = OpBuilder.reduce(kind, x, -1)
    fn.add_op(op)
    fn.output = op.outputs[0]
    return fn


@pytest.fixture(scope="module")
def c3b_input():
    rows, cols = 65536, 4096
    x = torch.randn(rows, cols, generator=torch.Generator().manual_seed(0))
    return x


@pytest.mark.parametrize("kind", ["sum", "max", "argmax", "softmax", "rms_norm"])
def test_reductions_full_65536x4096(cuda, c3b_input, kind):
    x = c3b_input
    rows, cols = x.shape
    fn = _row_fn(kind, rows, cols)
    prog = B200Compiler().compile(fn)
    assert [r["kernel"] for r in prog.spec.records] == ["rowreduce"]
    feed = {"x": x.to(cuda)}
    if kind == "rms_norm":
        feed["w"] = torch.ones(cols, device=cuda)
    got = prog.run(**feed)[0]
    ref = interp.run_function(fn, {k: v.cpu() for k, v in feed.items()})[0]
    if kind == "sum":
        exact = x.double().sum(-1)
        assert ((got.double() - exact).abs() <= 1e-6 * x.double().abs().sum(-1)).all()
        assert ((ref.double() - exact).abs() <= 1e-6 * x.double().abs().sum(-1)).all()
    elif kind in ("max", "argmax"):
        assert got.dtype == ref.dtype and torch.equal(got, ref)
    elif kind == "softmax":
        torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-9)
    else:
        torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-6)


# ----------------------------------------------------------------- models
def _close(got, ref, tol=2e-2):
    got, ref = got.float(), ref.float()
    bound = tol * (ref.abs().max() + ref.abs())
    err = (got - ref).abs()
    assert (err <= bound).all(), (err.max().item(), ref.abs().max().item())


def _runtime_inputs(ir, by_name):
    return {v.name: by_name[v.name] for v in ir.inputs if v.name not in ir.constants}


def test_vit_classifier_configured_shape(cuda):
    """All 27 layers at width 1152, 4 images (the 128-image batch's per-image work)."""
    B = 4
    imgs = workloads.preprocess_images(B, seed=5)
    pre = devproc.compile(workloads.vision_preprocess, imgs)
    pix = pre.run(images=imgs)[0]
    pre_ir = devproc.parse_ir(workloads.vision_preprocess, imgs)
    pix_ref = interp.run_function(pre_ir, {"images": imgs})[0]
    assert torch.equal(pix.view(torch.int16), pix_ref.view(torch.int16))

    # module on the CPU (weights drawn by the GPU's generator, which is faster)
    m = workloads.VitClassifier(logits=True, device=cuda).eval()
    prog = devproc.compile(m, pix)
    ir = prog.ir_function
    logits = prog.run(pix.to(cuda))[0]
    ref = interp.run_function(ir, _runtime_inputs(ir, {v.name: pix for v in ir.inputs}))[0]
    assert logits.shape == (B, 1000)
    _close(logits, ref)

    m.logits = False  # the configured pipeline ends in argmax
    prog_am = devproc.compile(m, pix)
    got = prog_am.run(pix.to(cuda))[0]
    top2 = ref.float().topk(2, -1).values
    decided = (top2[:, 0] - top2[:, 1]) > 2e-2 * ref.float().abs().max()
    assert torch.equal(got[decided].long(), ref.float().argmax(-1)[decided])


def test_pi05_policy_configured_shape(cuda):
    """One sample of the full policy: 27-layer encoder over 3 cameras, 18-layer
    Gemma-2B-shaped prefill over 816 tokens, 10 steps of the 18-layer expert."""
    imgs, ids, noise = workloads.pi05_inputs(1)
    pre = devproc.compile(workloads.vision_preprocess, imgs)
    pix = pre.run(images=imgs, to_cpu=False)[0]
    m = workloads.Pi05Policy(device=cuda).eval()
    prog = devproc.compile(m, pix, ids.to(cuda), noise.to(cuda))
    ir = prog.ir_function
    by_name = {"l_pixels_": pix, "l_text_ids_": ids.to(cuda), "l_noise_": noise.to(cuda)}
    got = prog.run(**_runtime_inputs(ir, by_name))[0]
    ref = interp.run_function(ir, {k: v.cpu() for k, v in _runtime_inputs(ir, by_name).items()})[0]
    assert got.shape == (1, 50, 32) and got.dtype == torch.float32
    _close(got, ref)
    # the denoised displacement itself (actions minus the starting noise), at the bf16 bar
    _close(got - noise, ref - noise)
