// GEMM entry point: validates the request and picks the kernel.
// bf16 × bf16 (B either [N, K] or [K, N]) and TF32 × TF32 (B as [N, K]) go
// to the tcgen05 tensor-core kernel when its TMA alignment rules hold (row
// and batch strides multiples of 16 bytes, 16-byte aligned bases); everything
// else (fp32, or odd strides) runs the FFMA kernel.  Both share one epilogue.
#include "dp_gemm_epilogue.cuh"

namespace dp {

int launch_gemm(const dp_gemm_params &p, const void *A, const void *B, void *C, const void *bias, const void *res,
                cudaStream_t s, void *sk_workspace, int64_t sk_bytes) {
  DP_REQUIRE(A && B && C, DP_ERR_ARG, "gemm: null A/B/C");
  DP_REQUIRE(p.M > 0 && p.N > 0 && p.K > 0 && p.batch > 0, DP_ERR_SHAPE, "gemm: sizes must be positive");
  DP_REQUIRE(p.lda >= p.K, DP_ERR_SHAPE, "gemm: lda < K");
  DP_REQUIRE(p.b_layout == DP_B_NK ? p.ldb >= p.K : p.ldb >= p.N, DP_ERR_SHAPE, "gemm: ldb too small");
  DP_REQUIRE(p.ldc >= p.N, DP_ERR_SHAPE, "gemm: ldc < N");
  DP_REQUIRE(p.M < (1ll << 31) / 1 && p.batch < 65536, DP_ERR_UNSUPPORTED, "gemm: M or batch too large");
  DP_REQUIRE(p.c_dtype == DP_F32 || p.c_dtype == DP_BF16 || p.c_dtype == DP_F16, DP_ERR_ARG,
             "gemm: C must be f32/bf16/f16");
  if (p.epilogue & DP_EPI_BIAS) DP_REQUIRE(bias != nullptr && dtype_bytes(p.bias_dtype) > 0, DP_ERR_ARG, "gemm: bias");
  DP_REQUIRE(!((p.epilogue & DP_EPI_RESIDUAL) && (p.epilogue & DP_EPI_MUL)), DP_ERR_ARG,
             "gemm: the residual is either added or multiplied, not both");
  if (p.epilogue & (DP_EPI_RESIDUAL | DP_EPI_MUL)) {
    DP_REQUIRE(res != nullptr && dtype_bytes(p.r_dtype) > 0, DP_ERR_ARG, "gemm: residual");
    DP_REQUIRE(p.ldr >= p.N, DP_ERR_SHAPE, "gemm: ldr < N");
  }
  const int acts = !!(p.epilogue & DP_EPI_RELU) + !!(p.epilogue & DP_EPI_GELU_ERF) +
                   !!(p.epilogue & DP_EPI_GELU_TANH) + !!(p.epilogue & DP_EPI_SILU);
  DP_REQUIRE(acts <= 1, DP_ERR_ARG, "gemm: at most one activation");
  DP_REQUIRE(p.batch2 <= 1 || p.batch % p.batch2 == 0, DP_ERR_SHAPE, "gemm: batch must be a multiple of batch2");
  if (p.epilogue & DP_EPI_SOFTMAX) {
    DP_REQUIRE(p.epilogue == DP_EPI_SOFTMAX, DP_ERR_ARG, "gemm: the softmax epilogue takes no other epilogue flag");
    DP_REQUIRE(p.N <= 256, DP_ERR_UNSUPPORTED, "gemm: the softmax epilogue needs N <= 256");
  }
  DP_REQUIRE(!(p.epilogue & DP_EPI_TF32SPLIT), DP_ERR_UNSUPPORTED,
             "gemm: the 3xTF32 operand store is an epilogue of dp_gemm_splitk_reduce only");
  if (p.epilogue & DP_EPI_ARGMAX)
    DP_REQUIRE(p.batch == 1 && !(p.epilogue & DP_EPI_SOFTMAX) &&
                   (reinterpret_cast<uintptr_t>(C) & 7) == 0,
               DP_ERR_ARG, "gemm: the argmax epilogue needs batch 1, no softmax and 8-byte aligned keys");
  const bool tf32 = p.a_dtype == DP_TF32 && p.b_dtype == DP_TF32;
  if ((p.a_dtype == DP_BF16 && p.b_dtype == DP_BF16) || (tf32 && p.b_layout == DP_B_NK)) {
    // operand rows and batch strides must be 16-byte multiples for TMA
    const int64_t v = tf32 ? 4 : 8;
    auto al = [](const void *q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
    const bool tc_ok = p.lda % v == 0 && p.ldb % v == 0 && p.stride_a % v == 0 && p.stride_b % v == 0 &&
                       p.stride_a2 % v == 0 && p.stride_b2 % v == 0 && al(A) && al(B);
    if (tc_ok) return launch_gemm_tc(p, A, B, C, bias, res, s, sk_workspace, sk_bytes);
  }
  DP_REQUIRE(!(p.epilogue & (DP_EPI_SOFTMAX | DP_EPI_ARGMAX)), DP_ERR_UNSUPPORTED,
             "gemm: the softmax and argmax epilogues run only on the tensor-core path (bf16 or TF32, 16-byte "
             "aligned operands)");
  return launch_gemm_simt(p, A, B, C, bias, res, s);
}

int launch_gemm_streamk(const dp_streamk_params &p, const void *A, const void *B, void *C, const void *bias,
                        const void *res, void *workspace, cudaStream_t s) {
  DP_REQUIRE(p.workspace_bytes >= 0 && (workspace != nullptr || p.workspace_bytes == 0), DP_ERR_ARG,
             "gemm_streamk: workspace_bytes without a workspace");
  return launch_gemm(p.gemm, A, B, C, bias, res, s, workspace, p.workspace_bytes);
}

}  // namespace dp

extern "C" int dp_gemm(const dp_gemm_params *p, const void *A, const void *B, void *C, const void *bias,
                       const void *residual, void *stream) {
  if (!p) return dp::set_error(DP_ERR_ARG, "dp_gemm: null params");
  return dp::launch_gemm(*p, A, B, C, bias, residual, dp::as_stream(stream));
}

extern "C" int dp_gemm_streamk_workspace(const dp_gemm_params *p, int64_t *bytes) {
  if (!p || !bytes) return dp::set_error(DP_ERR_ARG, "dp_gemm_streamk_workspace: null argument");
  DP_REQUIRE(p->M > 0 && p->N > 0 && p->batch > 0, DP_ERR_SHAPE, "dp_gemm_streamk_workspace: sizes must be positive");
  *bytes = dp::gemm_streamk_workspace_bound(*p);
  return DP_OK;
}

extern "C" int dp_gemm_streamk(const dp_streamk_params *p, const void *A, const void *B, void *C, const void *bias,
                               const void *residual, void *workspace, void *stream) {
  if (!p) return dp::set_error(DP_ERR_ARG, "dp_gemm_streamk: null params");
  return dp::launch_gemm_streamk(*p, A, B, C, bias, residual, workspace, dp::as_stream(stream));
}
