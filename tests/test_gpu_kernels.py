"""Parity of each sm_100a kernel with the CPU oracle, through the C ABI.

Tolerances (stated per test, following the pipeline's bar: bit-exact for
integer/index results, rtol 1e-4 for fp32, 2e-2 for bf16):
* preprocessing — bit-exact against the oracle's resize arithmetic;
* argmax / max / min / casts / gathers / transposes — exact;
* sum / mean — |Δ| ≤ 1e-6 · Σ|x| (a float32 summation-order bound);
* softmax — rtol 1e-5, atol 1e-8;  RMSNorm / LayerNorm — rtol 1e-4, atol 1e-5;
* fp32 GEMM — |Δ| ≤ 1e-4 · (|ref| + Σ_k |a_k b_k| / sqrt(K));
* bf16 results — rtol 2e-2, atol 2e-2.
"""

import numpy as np
import pytest
import torch

import devproc
from devproc_b200 import _native as N
from devproc_b200.ir.function import Function
from devproc_b200.ir.ops import OpBuilder
from devproc_b200.ir.types import TensorType
from devproc_b200 import workloads
from oracle import interp, preproc_np

pytestmark = pytest.mark.gpu

MEAN, STD = workloads.IMAGENET_MEAN, workloads.IMAGENET_STD


def _dt(t):
    return N.DTYPE_CODE[str(t.dtype).replace("torch.", "")]


def _sync():
    torch.cuda.synchronize()
    code, info = N.device_error()
    assert code == N.DP_DEVERR_NONE, (code, info)


# ---------------------------------------------------------------- preprocess
def _preproc_ref(x_nhwc_u8, oh, ow, normalize=True):
    y = preproc_np.resize_nhwc(x_nhwc_u8.numpy(), oh, ow)
    if normalize:
        y = ((y - np.asarray(MEAN, np.float32)).astype(np.float32) / np.asarray(STD, np.float32)).astype(np.float32)
    return torch.from_numpy(np.ascontiguousarray(y))


@pytest.mark.parametrize("B,H,W,OH,OW", [(4, 480, 640, 224, 224), (3, 96, 128, 56, 64), (2, 37, 53, 224, 99),
                                         (2, 1, 40, 3, 5), (2, 224, 224, 224, 224), (2, 17, 37, 8, 300),
                                         (2, 50, 32, 7, 2), (1, 64, 2048, 5, 1000), (2, 480, 640, 480, 640),
                                         (3, 100, 48, 300, 96)])
def test_preproc_nhwc_u8_to_nchw_bf16_bit_exact(cuda, B, H, W, OH, OW):
    x = workloads.preprocess_images(B, H, W, seed=B * H + W)
    out = torch.empty(B, 3, OH, OW, dtype=torch.bfloat16, device=cuda)
    p = N.PreprocParams(B, H, W, 3, OH, OW, N.DP_U8, N.DP_LAYOUT_NHWC, N.DP_BF16, N.DP_LAYOUT_NCHW, 1, 0)
    for c in range(3):
        p.mean[c], p.stdv[c] = MEAN[c], STD[c]
    N.preproc(p, x.to(cuda), out)
    _sync()
    ref = _preproc_ref(x, OH, OW).permute(0, 3, 1, 2).to(torch.bfloat16)
    assert torch.equal(out.cpu().view(torch.int16), ref.contiguous().view(torch.int16))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_preproc_fast_path_other_output_types(cuda, out_dtype):
    x = workloads.preprocess_images(3, 240, 320, seed=5)
    out = torch.empty(3, 3, 112, 160, dtype=out_dtype, device=cuda)
    p = N.PreprocParams(3, 240, 320, 3, 112, 160, N.DP_U8, N.DP_LAYOUT_NHWC, _dt(out), N.DP_LAYOUT_NCHW, 1, 0)
    for c in range(3):
        p.mean[c], p.stdv[c] = MEAN[c], STD[c]
    N.preproc(p, x.to(cuda), out)
    _sync()
    ref = _preproc_ref(x, 112, 160).permute(0, 3, 1, 2).to(out_dtype).contiguous()
    assert torch.equal(out.cpu(), ref)


def test_preproc_float_nchw_and_nhwc_out_bit_exact(cuda):
    g = torch.Generator().manual_seed(3)
    x = torch.rand(2, 3, 40, 72, generator=g) * 255  # NCHW fp32
    out = torch.empty(2, 31, 45, 3, dtype=torch.float32, device=cuda)  # NHWC fp32 out
    p = N.PreprocParams(2, 40, 72, 3, 31, 45, N.DP_F32, N.DP_LAYOUT_NCHW, N.DP_F32, N.DP_LAYOUT_NHWC, 0, 0)
    N.preproc(p, x.to(cuda), out)
    _sync()
    ref = preproc_np.resize_nhwc(x.permute(0, 2, 3, 1).numpy(), 31, 45)
    assert np.array_equal(out.cpu().numpy(), ref)


def test_preproc_full_batch_parity(cuda):
    """Full 256-image batch, every output element checked bit-exactly."""
    x = workloads.preprocess_images()
    out = torch.empty(256, 3, 224, 224, dtype=torch.bfloat16, device=cuda)
    p = N.PreprocParams(256, 480, 640, 3, 224, 224, N.DP_U8, N.DP_LAYOUT_NHWC, N.DP_BF16, N.DP_LAYOUT_NCHW, 1, 0)
    for c in range(3):
        p.mean[c], p.stdv[c] = MEAN[c], STD[c]
    N.preproc(p, x.to(cuda), out)
    _sync()
    got = out.cpu().view(torch.int16)
    for lo in range(0, 256, 32):
        ref = _preproc_ref(x[lo:lo + 32], 224, 224).permute(0, 3, 1, 2).to(torch.bfloat16)
        assert torch.equal(got[lo:lo + 32], ref.contiguous().view(torch.int16)), lo
    assert torch.isfinite(out.float()).all()


def test_preproc_rejects_bad_arguments(cuda):
    p = N.PreprocParams(1, 8, 8, 5, 4, 4, N.DP_U8, 0, N.DP_BF16, 1, 0, 0)
    with pytest.raises(N.DevProcError, match="4 channels"):
        N.preproc(p, torch.zeros(1, 8, 8, 5, dtype=torch.uint8, device=cuda),
                  torch.empty(1, 5, 4, 4, dtype=torch.bfloat16, device=cuda))


# ---------------------------------------------------------------- rowreduce
def _rr(kind, x, out_dtype, w=None, b=None, eps=0.0):
    rows, cols = x.shape
    if kind in (N.DP_RED_SOFTMAX, N.DP_RED_RMSNORM, N.DP_RED_LAYERNORM):
        out = torch.empty(rows, cols, dtype=out_dtype, device=x.device)
        ors = cols
    else:
        out = torch.empty(rows, dtype=out_dtype, device=x.device)
        ors = 1
    p = N.RowReduceParams(kind, _dt(x), _dt(out), int(w is not None), int(b is not None), 0, rows, cols, cols, ors,
                          eps, 0.0)
    N.rowreduce(p, x, out, w, b)
    _sync()
    return out.cpu()


@pytest.mark.parametrize("rows,cols", [(1024, 4096), (37, 1000), (8, 32000), (5, 3), (300, 8192 * 3 + 5)])
def test_value_reductions(cuda, rows, cols):
    g = torch.Generator().manual_seed(rows + cols)
    x = torch.randn(rows, cols, generator=g)
    xd = x.to(cuda)
    bound = 1e-6 * x.abs().sum(-1)
    s = _rr(N.DP_RED_SUM, xd, torch.float32)
    assert ((s - x.double().sum(-1).float()).abs() <= bound + 1e-7).all()
    m = _rr(N.DP_RED_MEAN, xd, torch.float32)
    assert ((m - x.double().mean(-1).float()).abs() <= bound / cols + 1e-7).all()
    assert torch.equal(_rr(N.DP_RED_MAX, xd, torch.float32), x.amax(-1))
    assert torch.equal(_rr(N.DP_RED_MIN, xd, torch.float32), x.amin(-1))
    assert torch.equal(_rr(N.DP_RED_ARGMAX, xd, torch.int64), x.argmax(-1))
    assert torch.equal(_rr(N.DP_RED_ARGMAX, xd, torch.int32), x.argmax(-1).int())


def test_argmax_ties_and_nan_first_index(cuda):
    x = torch.tensor([[1.0, 3.0, 3.0, 2.0] * 300, [float("nan")] * 1200, [-1.0] * 1200])
    x[1, :5] = 0.0
    x[1, 7] = float("nan")
    out = _rr(N.DP_RED_ARGMAX, x.to(cuda), torch.int64)
    assert out.tolist() == torch.argmax(x, -1).tolist() == [1, 5, 0]
    mx = _rr(N.DP_RED_MAX, x.to(cuda), torch.float32)
    assert torch.isnan(mx[1]) and mx[0] == 3.0


def test_argmax_infinities_and_ties_across_slots(cuda):
    """All -inf rows give index 0; equal maxima in different vector slots and
    lanes give the first index; +inf beats finite values."""
    x = torch.full((4, 4096), float("-inf"))
    x[1, 7], x[1, 2], x[1, 4000] = 5.0, 5.0, 5.0
    x[2] = torch.randn(4096)
    x[2, 129], x[2, 3] = float("inf"), float("inf")
    x[3] = 1.0
    out = _rr(N.DP_RED_ARGMAX, x.to(cuda), torch.int64)
    assert out.tolist() == torch.argmax(x, -1).tolist() == [0, 2, 3, 0]


def test_argmax_golden_vectors(cuda, golden):
    for case in ("argmax_small", "argmax_wide", "argmax_ties"):
        x = torch.from_numpy(golden[f"{case}/x"])
        out = _rr(N.DP_RED_ARGMAX, x.to(cuda), torch.int64)
        assert torch.equal(out, torch.from_numpy(golden[f"{case}/y"])), case


@pytest.mark.parametrize("rows,cols", [(1024, 4096), (37, 1000), (64, 512), (16, 20000), (3, 7), (300, 866), (64, 1003), (9, 3),
                                       (600, 1024), (1200, 2052), (700, 4092)])
def test_softmax_and_norms_fp32(cuda, rows, cols):
    g = torch.Generator().manual_seed(7 * rows + cols)
    x = torch.randn(rows, cols, generator=g) * 3
    w = torch.randn(cols, generator=g)
    b = torch.randn(cols, generator=g)
    xd = x.to(cuda)
    sm = _rr(N.DP_RED_SOFTMAX, xd, torch.float32)
    assert torch.allclose(sm, torch.softmax(x, -1), rtol=1e-5, atol=1e-8)
    rn = _rr(N.DP_RED_RMSNORM, xd, torch.float32, w=w.to(cuda), eps=1e-6)
    ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    assert torch.allclose(rn, ref, rtol=1e-4, atol=1e-5)
    ln = _rr(N.DP_RED_LAYERNORM, xd, torch.float32, w=w.to(cuda), b=b.to(cuda), eps=1e-5)
    assert torch.allclose(ln, torch.nn.functional.layer_norm(x, (cols,), w, b, 1e-5), rtol=1e-4, atol=1e-5)


def test_staged_rows_with_padded_strides(cuda):
    """fp32 rows staged through shared memory (enough rows for every SM),
    with input and output row strides larger than the row: each kind against
    torch, and the output padding left untouched."""
    g = torch.Generator().manual_seed(11)
    rows, cols, si, so = 900, 2048, 2056, 2064
    x = torch.randn(rows, si, generator=g) * 3
    w, b = torch.randn(cols, generator=g), torch.randn(cols, generator=g)
    xs = x[:, :cols]
    refs = {N.DP_RED_SOFTMAX: torch.softmax(xs, -1),
            N.DP_RED_RMSNORM: xs * torch.rsqrt(xs.pow(2).mean(-1, keepdim=True) + 1e-6) * w,
            N.DP_RED_LAYERNORM: torch.nn.functional.layer_norm(xs, (cols,), w, b, 1e-5)}
    for kind, ref in refs.items():
        out = torch.full((rows, so), float("nan"), device=cuda)
        has_w = int(kind != N.DP_RED_SOFTMAX)
        has_b = int(kind == N.DP_RED_LAYERNORM)
        eps = 1e-6 if kind == N.DP_RED_RMSNORM else 1e-5
        p = N.RowReduceParams(kind, N.DP_F32, N.DP_F32, has_w, has_b, 0, rows, cols, si, so, eps, 0.0)
        N.rowreduce(p, x.to(cuda), out, weight=w.to(cuda) if has_w else None, bias=b.to(cuda) if has_b else None)
        _sync()
        got = out.cpu()
        assert torch.allclose(got[:, :cols], ref, rtol=1e-4, atol=1e-5), kind
        assert torch.isnan(got[:, cols:]).all(), kind


@pytest.mark.parametrize("cols", [866, 50, 3, 1003])
def test_softmax_padded_rows_partial_vector(cuda, cols):
    """Attention-style rows: fp32 scores with rows padded to a multiple of 8,
    a column count that is not a whole number of vectors, bf16 output."""
    g = torch.Generator().manual_seed(cols)
    rows, stride = 257, (cols + 7) // 8 * 8
    x = torch.randn(rows, stride, generator=g) * 4
    out = torch.full((rows, stride), float("nan"), dtype=torch.bfloat16, device=cuda)
    p = N.RowReduceParams(N.DP_RED_SOFTMAX, N.DP_F32, N.DP_BF16, 0, 0, 0, rows, cols, stride, stride, 0.0, 0.0)
    N.rowreduce(p, x.to(cuda), out)
    _sync()
    ref = torch.softmax(x[:, :cols], -1)
    got = out.cpu()
    assert torch.allclose(got[:, :cols].float(), ref, rtol=1e-2, atol=1e-3)
    assert torch.isnan(got[:, cols:].float()).all()  # the pad is not written


def test_softmax_golden_vector(cuda, golden):
    x = torch.from_numpy(golden["softmax/x"])
    assert torch.allclose(_rr(N.DP_RED_SOFTMAX, x.to(cuda), torch.float32), torch.from_numpy(golden["softmax/y"]),
                          rtol=1e-5, atol=1e-8)


def test_norms_bf16(cuda):
    g = torch.Generator().manual_seed(11)
    x = torch.randn(256, 1152, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(1152, generator=g)).bfloat16()
    b = (0.1 * torch.randn(1152, generator=g)).bfloat16()
    ln = _rr(N.DP_RED_LAYERNORM, x.to(cuda), torch.bfloat16, w=w.to(cuda), b=b.to(cuda), eps=1e-6)
    ref = torch.nn.functional.layer_norm(x.float(), (1152,), w.float(), b.float(), 1e-6)
    assert torch.allclose(ln.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("rows,cols", [(300, 1152), (64, 264), (17, 2056), (5, 8), (1000, 2048)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_norms_16bit_row_kernel(cuda, rows, cols, dtype):
    """16-bit layernorm / rmsnorm (persistent warps, next row prefetched, weights in
    shared memory) against fp32 torch; rows not a multiple of 256 columns included."""
    g = torch.Generator().manual_seed(rows + cols)
    x = (3 * torch.randn(rows, cols, generator=g) + 1).to(dtype)
    w = (1 + 0.1 * torch.randn(cols, generator=g)).to(dtype)
    b = (0.1 * torch.randn(cols, generator=g)).to(dtype)
    ln = _rr(N.DP_RED_LAYERNORM, x.to(cuda), dtype, w=w.to(cuda), b=b.to(cuda), eps=1e-6)
    ref = torch.nn.functional.layer_norm(x.float(), (cols,), w.float(), b.float(), 1e-6)
    assert torch.allclose(ln.float(), ref, rtol=2e-2, atol=2e-2)
    rms = _rr(N.DP_RED_RMSNORM, x.to(cuda), dtype, w=w.to(cuda), eps=1e-6)
    ref = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert torch.allclose(rms.float(), ref, rtol=2e-2, atol=2e-2)


# ------------------------------------------------------------------- region
def _fn_of(build, *examples):
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


def _compile_run(fn, inputs):
    from devproc_b200.backend.b200 import B200Compiler
    prog = B200Compiler().compile(fn)
    out = prog.run(**inputs)
    return prog, out


def test_region_chain_with_broadcast(cuda):
    g = torch.Generator().manual_seed(5)
    x, y = torch.randn(333, 65, generator=g), torch.randn(65, generator=g)

    def build(a, b):
        o1 = OpBuilder.relu(a)
        o2 = OpBuilder.add(o1.outputs[0], b)
        o3 = OpBuilder.sigmoid(o2.outputs[0])
        return [o1, o2, o3]

    fn = _fn_of(build, x, y)
    prog, out = _compile_run(fn, {"x0": x, "x1": y})
    assert [r["kernel"] for r in prog.spec.records] == ["region"]
    ref = interp.run_function(fn, {"x0": x, "x1": y})[0]
    assert torch.allclose(out[0], ref, rtol=1e-6, atol=1e-7)


def test_region_golden_vectors(cuda, golden):
    for case, build in (("relu", OpBuilder.relu), ("normalize_f32", OpBuilder.normalize),
                        ("normalize_u8", OpBuilder.normalize)):
        x = torch.from_numpy(golden[f"{case}/x"])
        fn = _fn_of(lambda a: [build(a)], x)
        _, out = _compile_run(fn, {"x0": x})
        assert torch.equal(out[0], torch.from_numpy(golden[f"{case}/y"])), case
    x, x2 = torch.from_numpy(golden["add/x"]), torch.from_numpy(golden["add/x2"])
    fn = _fn_of(lambda a, b: [OpBuilder.add(a, b)], x, x2)
    _, out = _compile_run(fn, {"x0": x, "x1": x2})
    assert torch.equal(out[0], torch.from_numpy(golden["add/y"]))
    x = torch.from_numpy(golden["to_i32/x"])
    fn = _fn_of(lambda a: [OpBuilder.to(a, "int32")], x)
    _, out = _compile_run(fn, {"x0": x})
    assert torch.equal(out[0], torch.from_numpy(golden["to_i32/y"]))
    x = torch.from_numpy(golden["sigmoid/x"])
    fn = _fn_of(lambda a: [OpBuilder.sigmoid(a)], x)
    _, out = _compile_run(fn, {"x0": x})
    assert torch.allclose(out[0], torch.from_numpy(golden["sigmoid/y"]), rtol=1e-6, atol=1e-7)


def test_region_transpose_and_channel_normalize(cuda):
    x = workloads.preprocess_images(2, 12, 20, seed=9)

    def build(a):
        o1 = OpBuilder.normalize(a, MEAN, STD)
        o2 = OpBuilder.transpose(o1.outputs[0], (0, 3, 1, 2))
        o3 = OpBuilder.to(o2.outputs[0], "float16")
        return [o1, o2, o3]

    fn = _fn_of(build, x)
    _, out = _compile_run(fn, {"x0": x})
    ref = interp.run_function(fn, {"x0": x})[0]
    assert torch.equal(out[0].view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("shape", [(7, 33, 64), (3, 5, 12), (9, 4, 6), (2, 3, 7)])
def test_region_runs_of_each_width(cuda, shape):
    """Innermost extents divisible by 8, 4, 2 and 1 (run widths), bf16 and fp32
    vector paths, a broadcast operand and a permuted one, against the oracle."""
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(*shape, generator=g).bfloat16()
    y = torch.randn(shape[-1], generator=g)
    z = torch.randn(shape[1], shape[0], shape[2], generator=g)

    def build(a, b, c):
        o1 = OpBuilder.to(a, "float32")
        o2 = OpBuilder.add(o1.outputs[0], b)
        o3 = OpBuilder.transpose(c, (1, 0, 2))
        o4 = OpBuilder.binary("mul", o2.outputs[0], o3.outputs[0])
        o5 = OpBuilder.gelu(o4.outputs[0], approximate="tanh")
        o6 = OpBuilder.to(o5.outputs[0], "bfloat16")
        return [o1, o2, o3, o4, o5, o6]

    fn = _fn_of(build, x, y, z)
    _, out = _compile_run(fn, {"x0": x, "x1": y, "x2": z})
    ref = interp.run_function(fn, {"x0": x, "x1": y, "x2": z})[0]
    assert torch.allclose(out[0].float(), ref.float(), rtol=1e-2, atol=1e-2)


def test_region_pure_copy_moves_raw_int64(cuda):
    """A relayout copy of int64 values above 2^24 is exact (raw element moves,
    no float round trip)."""
    g = torch.Generator().manual_seed(3)
    x = torch.randint(-(1 << 40), 1 << 40, (6, 10, 16), generator=g, dtype=torch.int64)

    def build(a):
        o1 = OpBuilder.transpose(a, (1, 0, 2))
        o2 = OpBuilder.reshape(o1.outputs[0], (60, 16))
        return [o1, o2]

    fn = _fn_of(build, x)
    prog, out = _compile_run(fn, {"x0": x})
    assert kernels_of(prog) == ["region"]
    assert torch.equal(out[0], x.transpose(0, 1).reshape(60, 16))


def kernels_of(prog):
    return [r["kernel"] for r in prog.spec.records]


# --------------------------------------------------------------------- GEMM
def _gemm_bound(a, b_nk, ref):
    k = a.shape[-1]
    mag = (a.abs().double() @ b_nk.abs().double().T) / k ** 0.5
    return 1e-4 * (ref.abs().double() + mag)


@pytest.mark.parametrize("M,Nn,K", [(1024, 2048, 512), (37, 53, 29), (128, 32000, 512), (1, 10, 256)])
def test_gemm_fp32_linear_bias_gelu(cuda, M, Nn, K):
    g = torch.Generator().manual_seed(M + Nn + K)
    a = torch.randn(M, K, generator=g)
    w = torch.randn(Nn, K, generator=g) * 0.02
    bias = torch.randn(Nn, generator=g)
    c = torch.empty(M, Nn, device=cuda)
    p = N.GemmParams()
    p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.batch = M, Nn, K, K, K, Nn, 1
    p.a_dtype = p.b_dtype = p.c_dtype = p.bias_dtype = N.DP_F32
    p.b_layout = N.DP_B_NK
    p.epilogue = N.DP_EPI_BIAS | N.DP_EPI_GELU_ERF
    N.gemm(p, a.to(cuda), w.to(cuda), c, bias=bias.to(cuda))
    _sync()
    pre = (a.double() @ w.double().T + bias.double())
    ref = torch.nn.functional.gelu(pre)
    assert ((c.cpu().double() - ref).abs() <= _gemm_bound(a, w, ref) + 1e-6).all()


def test_gemm_fp32_matmul_kn_and_residual(cuda):
    g = torch.Generator().manual_seed(2)
    M, N_, K = 200, 72, 130
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N_, generator=g)
    r = torch.randn(M, N_, generator=g)
    c = torch.empty(M, N_, device=cuda)
    p = N.GemmParams()
    p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.ldr, p.batch = M, N_, K, K, N_, N_, N_, 1
    p.a_dtype = p.b_dtype = p.c_dtype = p.r_dtype = N.DP_F32
    p.b_layout = N.DP_B_KN
    p.epilogue = N.DP_EPI_RESIDUAL
    N.gemm(p, a.to(cuda), b.to(cuda), c, residual=r.to(cuda))
    _sync()
    ref = a.double() @ b.double() + r.double()
    assert ((c.cpu().double() - ref).abs() <= _gemm_bound(a, b.T, ref) + 1e-6).all()


def test_gemm_golden_vectors(cuda, golden):
    x, w = torch.from_numpy(golden["matmul/x"]), torch.from_numpy(golden["matmul/x2"])
    fn = _fn_of(lambda a, b: [OpBuilder.matmul(a, b)], x, w)
    _, out = _compile_run(fn, {"x0": x, "x1": w})
    assert torch.allclose(out[0], torch.from_numpy(golden["matmul/y"]), rtol=1e-5, atol=1e-5)
    x, w, b = (torch.from_numpy(golden[f"linear/{k}"]) for k in ("x", "x2", "b"))
    fn = _fn_of(lambda a, ww, bb: [OpBuilder.linear(a, ww, bb)], x, w, b)
    _, out = _compile_run(fn, {"x0": x, "x1": w, "x2": b})
    assert torch.allclose(out[0], torch.from_numpy(golden["linear/y"]), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("M,Nn,K", [(256, 512, 1024), (4096, 4096, 4096)])
def test_gemm_bf16(cuda, M, Nn, K):
    g = torch.Generator().manual_seed(M ^ Nn ^ K)
    a = torch.randn(M, K, generator=g).bfloat16()
    w = torch.randn(Nn, K, generator=g).bfloat16()
    c = torch.empty(M, Nn, device=cuda)
    p = N.GemmParams()
    p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.batch = M, Nn, K, K, K, Nn, 1
    p.a_dtype = p.b_dtype = N.DP_BF16
    p.c_dtype = N.DP_F32
    p.b_layout = N.DP_B_NK
    N.gemm(p, a.to(cuda), w.to(cuda), c)
    _sync()
    rows = slice(0, M) if M <= 512 else torch.arange(0, M, 61)
    ref = a[rows].float() @ w.float().T
    got = c.cpu()[rows]
    assert torch.allclose(got, ref, rtol=2e-2, atol=2e-2 * K ** 0.5 / 8)


def _bf16_gemm(cuda, M, Nn, K, epi=0, c_dtype=torch.float32, batch=1, bias=None, res=None, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(batch, M, K, generator=g).bfloat16()
    w = torch.randn(batch, Nn, K, generator=g).bfloat16()
    c = torch.empty(batch, M, Nn, dtype=c_dtype, device=cuda)
    p = N.GemmParams()
    p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.batch = M, Nn, K, K, K, Nn, batch
    p.stride_a, p.stride_b, p.stride_c = M * K, Nn * K, M * Nn
    p.a_dtype = p.b_dtype = N.DP_BF16
    p.c_dtype = _dt(c)
    p.b_layout = N.DP_B_NK
    p.epilogue = epi
    if bias is not None:
        p.bias_dtype = _dt(bias)
    if res is not None:
        p.r_dtype, p.ldr, p.stride_r = _dt(res), Nn, M * Nn
    N.gemm(p, a.to(cuda), w.to(cuda), c, bias=None if bias is None else bias.to(cuda),
           residual=None if res is None else res.to(cuda))
    _sync()
    return a, w, c.cpu()


@pytest.mark.parametrize("M,Nn,K", [(128, 256, 64), (256, 512, 1024), (37, 300, 72), (1, 10, 256), (300, 1000, 1152),
                                    # last column tile of at most 128 columns: N = 128 MMAs on CTA pairs
                                    (512, 1152, 1152), (300, 640, 512), (1000, 136, 256)])
def test_gemm_bf16_tensor_core_shapes(cuda, M, Nn, K):
    a, w, c = _bf16_gemm(cuda, M, Nn, K, seed=M + Nn)
    ref = a.float() @ w.float().transpose(-1, -2)
    assert torch.allclose(c, ref, rtol=1e-3, atol=1e-3 * K ** 0.5)


def test_gemm_bf16_epilogues_and_batch(cuda):
    g = torch.Generator().manual_seed(9)
    M, Nn, K = 200, 384, 256
    bias = torch.randn(Nn, generator=g).bfloat16()
    res = torch.randn(2, M, Nn, generator=g).bfloat16()
    a, w, c = _bf16_gemm(cuda, M, Nn, K, epi=N.DP_EPI_BIAS | N.DP_EPI_GELU_TANH | N.DP_EPI_RESIDUAL,
                         c_dtype=torch.bfloat16, batch=2, bias=bias, res=res, seed=3)
    acc = a.float() @ w.float().transpose(-1, -2) + bias.float()
    ref = torch.nn.functional.gelu(acc, approximate="tanh") + res.float()
    assert torch.allclose(c.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("M,Nn,K", [(256, 72, 256), (300, 500, 200), (128, 256, 64), (64, 1000, 136)])
def test_gemm_bf16_b_kn_tensor_core(cuda, M, Nn, K):
    """B as [K, N] (N contiguous, MN-major on the tensor cores), two-level batch."""
    g = torch.Generator().manual_seed(M * 7 + Nn)
    a = torch.randn(2, 3, M, K, generator=g).bfloat16()
    b = torch.randn(2, 3, K, Nn, generator=g).bfloat16()
    c = torch.empty(2, 3, M, Nn, dtype=torch.float32, device=cuda)
    p = N.GemmParams()
    p.M, p.N, p.K, p.lda, p.ldb, p.ldc = M, Nn, K, K, Nn, Nn
    p.batch, p.batch2 = 6, 3
    p.stride_a, p.stride_a2 = 3 * M * K, M * K
    p.stride_b, p.stride_b2 = 3 * K * Nn, K * Nn
    p.stride_c, p.stride_c2 = 3 * M * Nn, M * Nn
    p.a_dtype = p.b_dtype = N.DP_BF16
    p.c_dtype = N.DP_F32
    p.b_layout = N.DP_B_KN
    N.gemm(p, a.to(cuda), b.to(cuda), c)
    _sync()
    ref = a.float() @ b.float()
    assert torch.allclose(c.cpu(), ref, rtol=1e-3, atol=1e-3 * K ** 0.5)


@pytest.mark.parametrize("M,Nn,K", [(1024, 2048, 512), (300, 520, 128), (64, 32000, 512)])
def test_gemm_3xtf32_matches_fp32(cuda, M, Nn, K):
    """fp32 product on the tensor cores: one TF32 GEMM over [a_hi|a_hi|a_lo]·[b_hi|b_lo|b_hi]ᵀ
    agrees with an fp64 reference to fp32-level error (plain TF32 would not)."""
    g = torch.Generator().manual_seed(M + Nn)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(Nn, K, generator=g)

    def split(x):
        hi = (x.view(torch.int32) & -8192).view(torch.float32)
        return hi, x - hi

    ah, al = split(a)
    bh, bl = split(b)
    a3 = torch.cat([ah, ah, al], 1).contiguous()
    b3 = torch.cat([bh, bl, bh], 1).contiguous()
    c = torch.empty(M, Nn, dtype=torch.float32, device=cuda)
    p = N.GemmParams()
    p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.batch = M, Nn, 3 * K, 3 * K, 3 * K, Nn, 1
    p.a_dtype = p.b_dtype = N.DP_TF32
    p.c_dtype = N.DP_F32
    p.b_layout = N.DP_B_NK
    N.gemm(p, a3.to(cuda), b3.to(cuda), c)
    _sync()
    ref = a.double() @ b.double().T
    err = (c.cpu().double() - ref).abs() / (a.double().abs() @ b.double().abs().T)
    assert err.max() < 1e-5, err.max()  # plain TF32 (10-bit mantissas) gives ~1e-3


@pytest.mark.parametrize("c_dtype", [torch.bfloat16, torch.float32])
def test_gemm_multiply_epilogue(cuda, c_dtype):
    """C = (A·Bᵀ) ⊙ G with G an already computed operand (the up projection of
    a GeGLU times gelu(gate)), on the tensor-core path and the fp32 FFMA path."""
    g = torch.Generator().manual_seed(23)
    M, Nn, K = 300, 520, 256
    gate = torch.randn(M, Nn, generator=g).to(c_dtype)
    for in_dtype in (torch.bfloat16, torch.float32):
        a = torch.randn(M, K, generator=g).to(in_dtype)
        w = torch.randn(Nn, K, generator=g).to(in_dtype)
        c = torch.empty(M, Nn, dtype=c_dtype, device=cuda)
        p = N.GemmParams()
        p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.ldr, p.batch = M, Nn, K, K, K, Nn, Nn, 1
        p.a_dtype = p.b_dtype = _dt(a)
        p.c_dtype, p.r_dtype = _dt(c), _dt(gate)
        p.b_layout, p.epilogue = N.DP_B_NK, N.DP_EPI_MUL
        N.gemm(p, a.to(cuda), w.to(cuda), c, residual=gate.to(cuda))
        _sync()
        ref = (a.float() @ w.float().T) * gate.float()
        tol = 2e-2 if c_dtype == torch.bfloat16 or in_dtype == torch.bfloat16 else 1e-4
        assert torch.allclose(c.cpu().float(), ref, rtol=tol, atol=tol * ref.abs().max().item()), (in_dtype, c_dtype)


def test_gemm_bf16_batch_shared_b_and_residual(cuda):
    """Zero batch strides: one weight and one [M, N] residual shared by every
    batch (a position embedding added in the patch GEMM's epilogue)."""
    g = torch.Generator().manual_seed(17)
    batch, M, Nn, K = 3, 256, 384, 192
    a = torch.randn(batch, M, K, generator=g).bfloat16()
    w = torch.randn(Nn, K, generator=g).bfloat16()
    bias = torch.randn(Nn, generator=g).bfloat16()
    res = torch.randn(M, Nn, generator=g).bfloat16()
    for c_dtype in (torch.bfloat16, torch.float32):
        c = torch.empty(batch, M, Nn, dtype=c_dtype, device=cuda)
        p = N.GemmParams()
        p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.ldr, p.batch = M, Nn, K, K, K, Nn, Nn, batch
        p.stride_a, p.stride_b, p.stride_c, p.stride_r = M * K, 0, M * Nn, 0
        p.a_dtype = p.b_dtype = N.DP_BF16
        p.c_dtype, p.r_dtype, p.bias_dtype = _dt(c), N.DP_BF16, N.DP_BF16
        p.b_layout = N.DP_B_NK
        p.epilogue = N.DP_EPI_BIAS | N.DP_EPI_RESIDUAL
        N.gemm(p, a.to(cuda), w.to(cuda), c, bias=bias.to(cuda), residual=res.to(cuda))
        _sync()
        ref = a.float() @ w.float().T + bias.float() + res.float()
        assert torch.allclose(c.cpu().float(), ref, rtol=2e-2, atol=5e-2), c_dtype


def test_gemm_softmax_epilogue(cuda):
    """Row softmax of alpha·A·Bᵀ fused into the tensor-core epilogue, bf16 out, N < 256 masked."""
    g = torch.Generator().manual_seed(21)
    for (M, Nn, K) in [(256, 256, 72), (300, 200, 64), (200, 104, 64), (130, 136, 136)]:
        a = torch.randn(3, M, K, generator=g).bfloat16()
        b = torch.randn(3, Nn, K, generator=g).bfloat16()
        c = torch.empty(3, M, Nn, dtype=torch.bfloat16, device=cuda)
        p = N.GemmParams()
        p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.batch = M, Nn, K, K, K, Nn, 3
        p.stride_a, p.stride_b, p.stride_c = M * K, Nn * K, M * Nn
        p.a_dtype = p.b_dtype = p.c_dtype = N.DP_BF16
        p.b_layout, p.epilogue, p.alpha = N.DP_B_NK, N.DP_EPI_SOFTMAX, K ** -0.5
        N.gemm(p, a.to(cuda), b.to(cuda), c)
        _sync()
        ref = torch.softmax((a.float() @ b.float().transpose(-1, -2)) * K ** -0.5, -1)
        assert torch.allclose(c.cpu().float(), ref, rtol=2e-2, atol=2e-3)


# ---------------------------------------------------------------- embedding
def test_embedding_exact_and_index_error(cuda):
    g = torch.Generator().manual_seed(4)
    w = torch.randn(1000, 96, generator=g)
    ids = torch.randint(0, 1000, (7, 13), generator=g, dtype=torch.int32)
    out = torch.empty(7 * 13, 96, device=cuda)
    p = N.EmbeddingParams(ids.numel(), 1000, 96, N.DP_I32, N.DP_F32)
    N.embedding(p, ids.to(cuda), w.to(cuda), out)
    _sync()
    assert torch.equal(out.cpu().view(7, 13, 96), w[ids.long()])
    ids[3, 4] = 1000  # out of range
    N.embedding(p, ids.to(cuda), w.to(cuda), out)
    torch.cuda.synchronize()
    code, info = N.device_error()
    assert code == N.DP_DEVERR_INDEX and info == 3 * 13 + 4
    assert (out.cpu()[3 * 13 + 4] == 0).all()


# ---------------------------------------------------------------- attention
def _attn_ref(q, k, v, scale):
    g = q.shape[1] // k.shape[1]
    kk = k.float().repeat_interleave(g, 1)
    vv = v.float().repeat_interleave(g, 1)
    return torch.softmax((q.float() @ kk.transpose(-1, -2)) * scale, -1) @ vv


@pytest.mark.parametrize("B,Hk,g,L,S,D,Dv", [(2, 1, 8, 24, 50, 64, 64), (2, 1, 8, 50, 866, 256, 256),
                                              (1, 2, 4, 200, 300, 128, 128), (3, 4, 1, 256, 256, 72, 72),
                                              (1, 1, 1, 1, 1, 64, 64), (2, 2, 1, 130, 70, 256, 128),
                                              (32, 16, 1, 256, 256, 72, 72), (1, 1, 2, 64, 385, 96, 40),
                                              (2, 1, 1, 128, 129, 128, 8)])
def test_fused_attention(cuda, B, Hk, g, L, S, D, Dv):
    """Fused tcgen05 attention against fp32 torch: grouped-query heads stacked as rows,
    key counts not a multiple of the 64-key block, partial 128-row query tiles, head dims
    72 / 128 / 256, and the lazy running-max rescale (scores spread over a wide range)."""
    torch.manual_seed(B * 1000 + S)
    Hq = Hk * g
    q = (torch.randn(B, Hq, L, D) * 2).bfloat16()
    k = (torch.randn(B, Hk, S, D) * 2).bfloat16()
    v = torch.randn(B, Hk, S, Dv).bfloat16()
    scale = D ** -0.5
    o = torch.full((B, Hq, L, Dv), float("nan"), dtype=torch.bfloat16, device=cuda)
    p = N.AttentionParams()
    p.batch, p.heads_kv, p.group, p.L, p.S, p.D, p.Dv = B, Hk, g, L, S, D, Dv
    p.q_sb, p.q_sh, p.q_sl = Hq * L * D, L * D, D
    p.k_sb, p.k_sh, p.k_ss = Hk * S * D, S * D, D
    p.v_sb, p.v_sh, p.v_ss = Hk * S * Dv, S * Dv, Dv
    p.o_sb, p.o_sh, p.o_sl = Hq * L * Dv, L * Dv, Dv
    p.scale, p.dtype = scale, N.DP_BF16
    N.attention(p, q.to(cuda), k.to(cuda), v.to(cuda), o)
    _sync()
    ref = _attn_ref(q, k, v, scale)
    got = o.cpu().float()
    assert torch.allclose(got, ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item()), (got - ref).abs().max()


@pytest.mark.parametrize("D", [72, 256])
def test_fused_attention_rising_scores(cuda, D):
    """Scores that grow block after block (keys scaled up with their position),
    so the running max is raised and O / l rescaled on many blocks, with
    128-key blocks (D 72) and 64-key blocks (D 256)."""
    torch.manual_seed(D)
    B, H, L, S = 2, 2, 130, 700
    q = torch.randn(B, H, L, D).abs().bfloat16()
    k = (torch.randn(B, H, S, D).abs() * torch.linspace(0.1, 3.0, S)[:, None]).bfloat16()
    v = torch.randn(B, H, S, D).bfloat16()
    scale = D ** -0.5
    o = torch.empty(B, H, L, D, dtype=torch.bfloat16, device=cuda)
    p = N.AttentionParams()
    p.batch, p.heads_kv, p.group, p.L, p.S, p.D, p.Dv = B, H, 1, L, S, D, D
    p.q_sb, p.q_sh, p.q_sl = H * L * D, L * D, D
    p.k_sb, p.k_sh, p.k_ss = H * S * D, S * D, D
    p.v_sb, p.v_sh, p.v_ss = H * S * D, S * D, D
    p.o_sb, p.o_sh, p.o_sl = H * L * D, L * D, D
    p.scale, p.dtype = scale, N.DP_BF16
    N.attention(p, q.to(cuda), k.to(cuda), v.to(cuda), o)
    _sync()
    ref = _attn_ref(q, k, v, scale)
    assert torch.allclose(o.cpu().float(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())


@pytest.mark.parametrize("D,scale", [(256, -0.0625), (72, -0.125), (256, 0.0), (72, 0.0)])
def test_fused_attention_negative_and_zero_scale(cuda, D, scale):
    """The kernel takes the row max on raw scores and folds the scale into the
    exponent: a negative scale (max of the negated scores) and a zero scale
    (uniform weights over the valid keys, the partial last block masked) still
    match softmax(scale · Q·Kᵀ)·V."""
    torch.manual_seed(7 + D)
    B, H, L, S = 1, 2, 130, 201
    q = torch.randn(B, H, L, D).bfloat16()
    k = torch.randn(B, H, S, D).bfloat16()
    v = torch.randn(B, H, S, D).bfloat16()
    o = torch.empty(B, H, L, D, dtype=torch.bfloat16, device=cuda)
    p = N.AttentionParams()
    p.batch, p.heads_kv, p.group, p.L, p.S, p.D, p.Dv = B, H, 1, L, S, D, D
    p.q_sb, p.q_sh, p.q_sl = H * L * D, L * D, D
    p.k_sb, p.k_sh, p.k_ss = H * S * D, S * D, D
    p.v_sb, p.v_sh, p.v_ss = H * S * D, S * D, D
    p.o_sb, p.o_sh, p.o_sl = H * L * D, L * D, D
    p.scale, p.dtype = scale, N.DP_BF16
    N.attention(p, q.to(cuda), k.to(cuda), v.to(cuda), o)
    _sync()
    ref = _attn_ref(q, k, v, scale)
    got = o.cpu().float()
    assert torch.isfinite(got).all()
    assert torch.allclose(got, ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item()), (got - ref).abs().max()


def test_fused_attention_token_major_output(cuda):
    """One query head per key head with the output stored token-major [B, L, H, Dv]
    (the layout the following reshape reads for free) and strided q / k / v column
    blocks of one fused projection."""
    torch.manual_seed(5)
    B, H, L, D = 2, 4, 96, 72
    qkv = torch.randn(B, L, 3 * H * D).bfloat16()
    q = qkv[..., :H * D].reshape(B, L, H, D).transpose(1, 2)
    k = qkv[..., H * D:2 * H * D].reshape(B, L, H, D).transpose(1, 2)
    v = qkv[..., 2 * H * D:].reshape(B, L, H, D).transpose(1, 2)
    d = qkv.to(cuda)
    out = torch.empty(B, L, H, D, dtype=torch.bfloat16, device=cuda)
    p = N.AttentionParams()
    p.batch, p.heads_kv, p.group, p.L, p.S, p.D, p.Dv = B, H, 1, L, L, D, D
    row = 3 * H * D
    p.q_sb, p.q_sh, p.q_sl = L * row, D, row
    p.k_sb, p.k_sh, p.k_ss = L * row, D, row
    p.v_sb, p.v_sh, p.v_ss = L * row, D, row
    p.o_sb, p.o_sh, p.o_sl = L * H * D, D, H * D
    p.scale, p.dtype = D ** -0.5, N.DP_BF16
    es = d.element_size()
    N.attention(p, d.data_ptr(), d.data_ptr() + H * D * es, d.data_ptr() + 2 * H * D * es, out)
    _sync()
    ref = _attn_ref(q, k, v, D ** -0.5).transpose(1, 2)
    assert torch.allclose(out.cpu().float(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())


# ---------------------------------------------------------------- split-K
class _LinearGelu(torch.nn.Module):
    def __init__(self, k, n, dtype):
        super().__init__()
        self.lin = torch.nn.Linear(k, n).to(dtype)

    def forward(self, x, r):
        return torch.nn.functional.gelu(self.lin(x)) + r


@pytest.mark.parametrize("dtype,M,K,Nn", [(torch.float32, 1024, 2048, 512), (torch.float32, 1024, 512, 2048),
                                          (torch.bfloat16, 256, 8192, 512)])
def test_split_k_linear_matches_fp64(cuda, dtype, M, K, Nn):
    """Linears with few output tiles and a long K run as a batched GEMM over K
    slices plus a reduce that applies bias, GELU and the residual.  fp32
    (3xTF32) within rtol 1e-4 of the fp64 product; bf16 within the bf16 bar."""
    torch.manual_seed(0)
    m = _LinearGelu(K, Nn, dtype).eval()
    x = torch.randn(M, K).to(dtype)
    r = torch.randn(M, Nn).to(dtype)
    prog = devproc.compile(m, x, r)
    kinds = [rec["kernel"] for rec in prog.spec.records]
    assert "splitk" in kinds, prog.describe()
    got = prog.run(x, r)[0].double()
    w, b = m.lin.weight.double(), m.lin.bias.double()
    ref = torch.nn.functional.gelu(x.double() @ w.T + b) + r.double()
    mag = (x.double().abs() @ w.abs().T) + b.abs() + r.double().abs()
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert ((got - ref).abs() <= tol * mag).all(), ((got - ref).abs() / mag).max()
    again = prog.run(x, r)[0]
    assert torch.equal(again.double(), got)  # slices are summed in a fixed order


# ------------------------------------------------------- stream-K GEMM
@pytest.mark.parametrize("M,Nn,K,batch,c_dtype,epi,ldc_pad", [
    # the action expert's down projection: 52 pair tiles for 74 CTA pairs
    (3200, 1024, 4096, 1, torch.bfloat16, N.DP_EPI_BIAS | N.DP_EPI_GELU_TANH | N.DP_EPI_RESIDUAL, 0),
    (3200, 1024, 4096, 1, torch.float32, 0, 0),
    # single-CTA tiles: 79 tiles for 148 CTAs
    (100, 20000, 2048, 1, torch.bfloat16, N.DP_EPI_BIAS, 0),
    # batched, ragged edges, output rows not 16-byte multiples (no TMA store)
    (1000, 600, 3000, 3, torch.bfloat16, N.DP_EPI_RESIDUAL, 1),
])
def test_streamk_gemm_matches_fp64(cuda, M, Nn, K, batch, c_dtype, epi, ldc_pad):
    """dp_gemm_streamk: the K stages of the tiles past the last full wave are
    dealt out over every CTA group and the tile-ending group adds the earlier
    partials.  Checked against the fp64 product (bf16 bar), bit-identical on
    a second run (partials are added in a fixed order), and the per-tile
    arrival counters show the split really ran."""
    g = torch.Generator().manual_seed(M + K + batch)
    a = torch.randn(batch, M, K, generator=g).bfloat16().to(cuda)
    w = (torch.randn(batch, Nn, K, generator=g) * 0.05).bfloat16().to(cuda)
    bias = torch.randn(Nn, generator=g).to(c_dtype).to(cuda)
    ldc = Nn + ldc_pad
    res = torch.randn(batch, M, ldc, generator=g).to(c_dtype).to(cuda)
    c = torch.zeros(batch, M, ldc, dtype=c_dtype, device=cuda)
    p = N.GemmParams()
    p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.ldr, p.batch = M, Nn, K, K, K, ldc, ldc, batch
    p.stride_a, p.stride_b, p.stride_c, p.stride_r = M * K, Nn * K, M * ldc, M * ldc
    p.a_dtype = p.b_dtype = N.DP_BF16
    p.c_dtype = p.r_dtype = p.bias_dtype = _dt(c)
    p.b_layout = N.DP_B_NK
    p.epilogue = epi
    sp = N.StreamKParams()
    sp.gemm, sp.workspace_bytes = p, N.gemm_streamk_workspace(p)
    ws = torch.zeros(sp.workspace_bytes, dtype=torch.uint8, device=cuda)
    N.gemm_streamk(sp, a, w, c, ws, bias=bias, residual=res)
    _sync()
    counters = ws[:4 * 64].view(torch.int32).cpu()
    assert int(counters.max()) > 0, "the stream-K split did not run"
    acc = a.double() @ w.double().transpose(-1, -2)
    mag = a.double().abs() @ w.double().abs().transpose(-1, -2)
    if epi & N.DP_EPI_BIAS:
        acc = acc + bias.double()
        mag = mag + bias.double().abs()
    if epi & N.DP_EPI_GELU_TANH:
        acc = torch.nn.functional.gelu(acc, approximate="tanh")
    if epi & N.DP_EPI_RESIDUAL:
        acc = acc + res[..., :Nn].double()
        mag = mag + res[..., :Nn].double().abs()
    got = c[..., :Nn].double()
    tol = 2e-2 if c_dtype == torch.bfloat16 else 1e-3
    assert ((got - acc).abs() <= tol * mag + 1e-3).all(), ((got - acc).abs() / (mag + 1e-3)).max()
    if ldc_pad:
        assert (c[..., Nn:] == 0).all()  # padding columns untouched
    first = c.clone()
    N.gemm_streamk(sp, a, w, c, ws, bias=bias, residual=res)
    _sync()
    assert torch.equal(c, first)
    # the same call without a workspace runs whole tiles and agrees within rounding
    whole = torch.zeros_like(c)
    N.gemm(p, a, w, whole, bias=bias, residual=res)
    _sync()
    assert ((whole[..., :Nn].double() - got).abs() <= tol * mag + 1e-3).all()


def test_streamk_linear_program_matches_fp64(cuda):
    """With stream-K switched on, a compiled bf16 linear + GELU + residual with
    a ragged last wave runs as one stream-K record; fp64 bar as for the other
    bf16 linears."""
    from devproc_b200.backend.b200.lowering import Lowerer
    torch.manual_seed(1)
    m = _LinearGelu(4096, 1024, torch.bfloat16).eval()
    x = torch.randn(3200, 4096).to(torch.bfloat16)
    r = torch.randn(3200, 1024).to(torch.bfloat16)
    Lowerer.use_streamk = True
    try:
        prog = devproc.compile(m, x, r)
    finally:
        Lowerer.use_streamk = False
    assert [rec["kernel"] for rec in prog.spec.records] == ["gemm_sk"], prog.describe()
    got = prog.run(x, r)[0].double()
    w, b = m.lin.weight.double(), m.lin.bias.double()
    ref = torch.nn.functional.gelu(x.double() @ w.T + b) + r.double()
    mag = (x.double().abs() @ w.abs().T) + b.abs() + r.double().abs()
    assert ((got - ref).abs() <= 2e-2 * mag).all(), ((got - ref).abs() / mag).max()
    assert torch.equal(prog.run(x, r)[0].double(), got)


# --------------------------------------------- 3xTF32 operands written by their producer
def _tf32_split(x):
    hi = (x.contiguous().view(torch.int32) & -8192).view(torch.float32)
    return torch.cat([hi, hi, x - hi], dim=-1)


def test_splitk_reduce_and_layernorm_store_3xtf32_operands(cuda):
    """DP_EPI_TF32SPLIT on the split-K reduce and out_split on the fp32
    LayerNorm store [hi | hi | lo] rows: bit-identical to the plain result
    split afterwards (hi = the value with the low 13 mantissa bits cleared)."""
    g = torch.Generator().manual_seed(5)
    M, Nn, S = 300, 520, 3
    ws = torch.randn(S, M, Nn, generator=g).to(cuda)
    bias = torch.randn(Nn, generator=g).to(cuda)
    sp = N.SplitKParams()
    sp.gemm.M, sp.gemm.N, sp.gemm.K, sp.gemm.batch = M, Nn, 64, 1
    sp.gemm.c_dtype = sp.gemm.bias_dtype = N.DP_F32
    sp.gemm.epilogue = N.DP_EPI_BIAS | N.DP_EPI_GELU_ERF
    sp.gemm.ldc = Nn
    sp.splits, sp.slice_stride = S, M * Nn
    plain = torch.empty(M, Nn, device=cuda)
    N.gemm_splitk_reduce(sp, ws, plain, bias=bias)
    sp.gemm.epilogue |= N.DP_EPI_TF32SPLIT
    sp.gemm.ldc = 3 * Nn
    split = torch.empty(M, 3 * Nn, device=cuda)
    N.gemm_splitk_reduce(sp, ws, split, bias=bias)
    _sync()
    assert torch.equal(split.cpu(), _tf32_split(plain.cpu()))

    x = torch.randn(M, Nn, generator=g).to(cuda)
    w = torch.randn(Nn, generator=g).to(cuda)
    b = torch.randn(Nn, generator=g).to(cuda)
    p = N.RowReduceParams()
    p.kind, p.in_dtype, p.out_dtype = N.DP_RED_LAYERNORM, N.DP_F32, N.DP_F32
    p.has_weight, p.has_bias, p.rows, p.cols, p.in_row_stride, p.out_row_stride = 1, 1, M, Nn, Nn, Nn
    p.eps = 1e-5
    ln = torch.empty(M, Nn, device=cuda)
    N.rowreduce(p, x, ln, weight=w, bias=b)
    p.out_split, p.out_row_stride = 1, 3 * Nn
    ln3 = torch.empty(M, 3 * Nn, device=cuda)
    N.rowreduce(p, x, ln3, weight=w, bias=b)
    _sync()
    assert torch.equal(ln3.cpu(), _tf32_split(ln.cpu()))


# ------------------------------------------------------- argmax epilogue
class _LinearArgmax(torch.nn.Module):
    def __init__(self, k, n, dtype):
        super().__init__()
        self.lin = torch.nn.Linear(k, n).to(dtype)

    def forward(self, x):
        return self.lin(x).argmax(-1).to(torch.int32)


@pytest.mark.parametrize("dtype,M,K,Nn", [(torch.float32, 512, 512, 3000), (torch.bfloat16, 300, 256, 1000)])
def test_argmax_epilogue_matches_oracle_and_breaks_ties_first(cuda, dtype, M, K, Nn):
    """linear -> argmax lowers to one GEMM whose epilogue folds each row into a
    (value, first column) key; the logits are never stored.  Indices must equal
    the oracle's (torch.argmax of the same-dtype logits) on every row whose
    top-2 gap exceeds the float bar, and columns with identical logits (rows of
    the weight duplicated, a large shared bias) must give the first column."""
    torch.manual_seed(1)
    m = _LinearArgmax(K, Nn, dtype).eval()
    x = torch.randn(M, K).to(dtype)
    prog = devproc.compile(m, x)
    assert [r["kernel"] for r in prog.spec.records][-3:] == ["argmax_keys", "gemm", "argmax_keys"]
    ir = devproc.from_torch(m, x, backend="ir")
    name = [v.name for v in ir.inputs if v.name not in ir.constants][0]
    got = prog.run(x)[0]
    ref = interp.run_function(ir, {name: x})[0]
    logits = (x.double() @ m.lin.weight.double().T + m.lin.bias.double())
    top2 = logits.topk(2, -1).values
    decided = (top2[:, 0] - top2[:, 1]) > (1e-4 if dtype == torch.float32 else 2e-2) * logits.abs().max()
    assert decided.float().mean() > 0.5
    assert got.dtype == torch.int32 and torch.equal(got[decided], ref[decided])
    with torch.no_grad():  # columns 7, 11 and 700 identical and dominant: every row picks 7
        m.lin.weight[11] = m.lin.weight[7]
        m.lin.weight[700] = m.lin.weight[7]
        m.lin.bias[7] = m.lin.bias[11] = m.lin.bias[700] = 1000.0
    prog = devproc.compile(m, x)
    assert (prog.run(x)[0] == 7).all()
