// Helper kernels of the GEMM: the split-K reduction and the argmax keys.
//
// Split-K reduction: the second half of a GEMM whose K range was split.
// A GEMM with few output tiles and a long K (the fp32 token pipeline's
// M = 1024 linears: 8 or 32 CTA-pair tiles for 74 pairs) leaves most SMs idle
// if each tile walks all of K.  The lowering then runs it as a batched GEMM
// over S slices of K, each writing raw fp32 partial products to slice s of a
// workspace [S, M, N], and this kernel sums the slices in slice order (the
// same bits every run), applies the GEMM's epilogue (alpha, bias, activation,
// residual or gate operand) and writes C in its dtype.
//
// Argmax keys: a GEMM with the DP_EPI_ARGMAX epilogue reduces each row of its
// result to one 64-bit key by atomicMax; argmax_keys_kernel zeroes the keys
// before it and turns them into column indices after it.
#include "dp_gemm_epilogue.cuh"

namespace dpk_splitk {

__global__ void __launch_bounds__(256) splitk_reduce_kernel(dp_splitk_params sp, const float *__restrict__ ws,
                                                             void *C, const void *bias, const void *res) {
  dp::pdl_trigger();
  dp::pdl_wait();
  const dp_gemm_params &p = sp.gemm;
  const dp::Epilogue ep(p, C, bias, res, 0);
  const int64_t nq = (p.N + 3) / 4;  // column quads per row
  const int64_t total = p.M * nq;
  const bool vec = (p.N % 4) == 0 && (sp.slice_stride % 4) == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / nq, n = (i - m * nq) * 4;
    const int64_t off = m * p.N + n;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (vec) {
      for (int64_t s = 0; s < sp.splits; ++s) {
        const float4 x = __ldg(reinterpret_cast<const float4 *>(ws + s * sp.slice_stride + off));
        v[0] += x.x;
        v[1] += x.y;
        v[2] += x.z;
        v[3] += x.w;
      }
    } else {
      for (int64_t s = 0; s < sp.splits; ++s)
        for (int j = 0; j < 4; ++j)
          if (n + j < p.N) v[j] += ws[s * sp.slice_stride + off + j];
    }
    ep.store4(m, n, v[0], v[1], v[2], v[3]);
  }
}

__global__ void argmax_keys_kernel(dp_argmax_keys_params p, unsigned long long *keys, void *out) {
  dp::pdl_trigger();
  dp::pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < p.n; i += (int64_t)gridDim.x * blockDim.x) {
    if (p.mode == 0) {
      keys[i] = 0ull;
    } else {
      const int64_t col = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[i] & 0xFFFFFFFFull));
      if (p.out_dtype == DP_I32)
        static_cast<int32_t *>(out)[i] = (int32_t)col;
      else
        static_cast<long long *>(out)[i] = col;
    }
  }
}

}  // namespace dpk_splitk

namespace dp {

int launch_splitk_reduce(const dp_splitk_params &sp, const void *ws, void *C, const void *bias, const void *res,
                         cudaStream_t s) {
  const dp_gemm_params &p = sp.gemm;
  DP_REQUIRE(ws && C, DP_ERR_ARG, "splitk: null workspace or C");
  DP_REQUIRE(p.M > 0 && p.N > 0 && sp.splits > 0 && p.batch == 1, DP_ERR_SHAPE,
             "splitk: M, N and splits must be positive, batch 1");
  DP_REQUIRE(sp.slice_stride >= p.M * p.N, DP_ERR_SHAPE, "splitk: slice_stride < M * N");
  DP_REQUIRE(p.ldc >= p.N, DP_ERR_SHAPE, "splitk: ldc < N");
  DP_REQUIRE(p.c_dtype == DP_F32 || p.c_dtype == DP_BF16 || p.c_dtype == DP_F16, DP_ERR_ARG,
             "splitk: C must be f32/bf16/f16");
  DP_REQUIRE(!(p.epilogue & (DP_EPI_SOFTMAX | DP_EPI_ARGMAX)), DP_ERR_UNSUPPORTED,
             "splitk: no softmax or argmax epilogue");
  if (p.epilogue & DP_EPI_TF32SPLIT)
    DP_REQUIRE(p.c_dtype == DP_F32 && p.ldc >= 3 * p.N, DP_ERR_ARG,
               "splitk: the 3xTF32 operand store needs fp32 C with ldc >= 3 N");
  if (p.epilogue & DP_EPI_BIAS) DP_REQUIRE(bias != nullptr, DP_ERR_ARG, "splitk: bias");
  if (p.epilogue & (DP_EPI_RESIDUAL | DP_EPI_MUL)) DP_REQUIRE(res != nullptr, DP_ERR_ARG, "splitk: residual");
  const int64_t quads = p.M * ((p.N + 3) / 4);
  int64_t blocks = (quads + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  dp::launch_k(dpk_splitk::splitk_reduce_kernel, (int)blocks, 256, 0, s, sp, static_cast<const float *>(ws), C, bias, res);
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

int launch_argmax_keys(const dp_argmax_keys_params &p, void *keys, void *out, cudaStream_t s) {
  DP_REQUIRE(keys != nullptr && p.n > 0, DP_ERR_ARG, "argmax_keys: null keys or empty");
  DP_REQUIRE(p.mode == 0 || p.mode == 1, DP_ERR_ARG, "argmax_keys: mode is 0 (clear) or 1 (indices)");
  if (p.mode == 1) {
    DP_REQUIRE(out != nullptr, DP_ERR_ARG, "argmax_keys: null output");
    DP_REQUIRE(p.out_dtype == DP_I32 || p.out_dtype == DP_I64, DP_ERR_ARG, "argmax_keys: indices are i32 or i64");
  }
  int64_t blocks = (p.n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  dp::launch_k(dpk_splitk::argmax_keys_kernel, (int)blocks, 256, 0, s, p, static_cast<unsigned long long *>(keys), out);
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

}  // namespace dp

extern "C" int dp_argmax_keys(const dp_argmax_keys_params *p, void *keys, void *out, void *stream) {
  if (!p) return dp::set_error(DP_ERR_ARG, "dp_argmax_keys: null params");
  return dp::launch_argmax_keys(*p, keys, out, dp::as_stream(stream));
}

extern "C" int dp_gemm_splitk_reduce(const dp_splitk_params *p, const void *workspace, void *C, const void *bias,
                                     const void *residual, void *stream) {
  if (!p) return dp::set_error(DP_ERR_ARG, "dp_gemm_splitk_reduce: null params");
  return dp::launch_splitk_reduce(*p, workspace, C, bias, residual, dp::as_stream(stream));
}
