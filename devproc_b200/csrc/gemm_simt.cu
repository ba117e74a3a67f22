// FP32-exact GEMM on the CUDA cores (FFMA), for fp32 graphs whose tolerance
// (rtol 1e-4) TF32 tensor cores cannot meet, e.g. the fp32 token pipeline.
//
// Replaces the reference's matmul_kernel / linear_kernel for fp32 inputs
// (src/devproc/backend/triton/templates/matmul.py:24-224), whose K loop
// masked out every K block after the first (the mask compares the already
// advanced offs_k against K - k*BLOCK_K, matmul.py:88-99) and whose tl.dot
// on fp32 runs as TF32.
//
// Tile 128×128×8, 256 threads, 8×8 outputs per thread held in registers,
// two shared-memory buffers with the next tile prefetched into registers
// while the current one is multiplied.  Each output accumulates over K in
// order with fmaf, so its rounding error grows like sqrt(K)·eps.
#include "dp_gemm_epilogue.cuh"

namespace dpk_sgemm {

constexpr int BM = 128, BN = 128, BK = 8, kThreads = 256;

template <typename T>
__device__ __forceinline__ void load4(const T *p, bool vec, int64_t valid, float (&v)[4]) {
  if (vec && valid >= 4) {
    if constexpr (sizeof(T) == 4) {
      const float4 q = __ldg(reinterpret_cast<const float4 *>(p));
      v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    } else {
      const uint2 q = __ldg(reinterpret_cast<const uint2 *>(p));
      const T *e = reinterpret_cast<const T *>(&q);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = to_f32(e[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = j < valid ? to_f32(p[j]) : 0.0f;
  }
}

// B_NK: B is [N, K] (K contiguous); otherwise [K, N] (N contiguous).
template <typename TA, typename TB, bool B_NK>
__global__ void __launch_bounds__(kThreads) sgemm_kernel(dp_gemm_params p, const TA *__restrict__ A,
                                                         const TB *__restrict__ B, void *C,
                                                         const void *bias, const void *res, bool a_vec,
                                                         bool b_vec) {
  dp::pdl_trigger();
  dp::pdl_wait();
  __shared__ __align__(16) float As[2][BK][BM + 4];
  __shared__ __align__(16) float Bs[2][BK][BN + 4];
  const int64_t bz = blockIdx.z;
  {
    const int64_t b2 = p.batch2 > 1 ? p.batch2 : 1;
    const int64_t zo = bz / b2, zi = bz - zo * b2;
    A += zo * p.stride_a + zi * p.stride_a2;
    B += zo * p.stride_b + zi * p.stride_b2;
  }
  const int tid = threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int tx = tid % 16, ty = tid / 16;

  // Global → register staging coordinates.
  const int a_row = tid / 2, a_k = (tid % 2) * 4;
  const int bnk_row = tid / 2, bnk_k = (tid % 2) * 4;  // B as [N, K]
  const int bkn_k = tid / 32, bkn_n = (tid % 32) * 4;  // B as [K, N]

  float ra[4], rb[4];
  auto fetch = [&](int64_t k0) {
    {
      const int64_t m = m0 + a_row, k = k0 + a_k;
      if (m < p.M && k < p.K)
        load4(A + m * p.lda + k, a_vec, p.K - k, ra);
      else
        ra[0] = ra[1] = ra[2] = ra[3] = 0.0f;
    }
    if (B_NK) {
      const int64_t n = n0 + bnk_row, k = k0 + bnk_k;
      if (n < p.N && k < p.K)
        load4(B + n * p.ldb + k, b_vec, p.K - k, rb);
      else
        rb[0] = rb[1] = rb[2] = rb[3] = 0.0f;
    } else {
      const int64_t k = k0 + bkn_k, n = n0 + bkn_n;
      if (k < p.K && n < p.N)
        load4(B + k * p.ldb + n, b_vec, p.N - n, rb);
      else
        rb[0] = rb[1] = rb[2] = rb[3] = 0.0f;
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int j = 0; j < 4; ++j) As[buf][a_k + j][a_row] = ra[j];
    if (B_NK) {
#pragma unroll
      for (int j = 0; j < 4; ++j) Bs[buf][bnk_k + j][bnk_row] = rb[j];
    } else {
      *reinterpret_cast<float4 *>(&Bs[buf][bkn_k][bkn_n]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  const int64_t ktiles = (p.K + BK - 1) / BK;
  fetch(0);
  stash(0);
  __syncthreads();
  for (int64_t t = 0; t < ktiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ktiles) fetch((t + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (t + 1 < ktiles) {
      stash(buf ^ 1);
      __syncthreads();
    }
  }

  dp::Epilogue ep(p, C, bias, res, bz);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= p.M) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t n = n0 + h * 64 + tx * 4;
      ep.store4(m, n, acc[i][h * 4 + 0], acc[i][h * 4 + 1], acc[i][h * 4 + 2], acc[i][h * 4 + 3]);
    }
  }
}

template <typename TA, typename TB>
int launch_typed(const dp_gemm_params &p, const void *A, const void *B, void *C, const void *bias,
                 const void *res, cudaStream_t s) {
  const int esz = sizeof(TA);
  auto al = [](const void *q, int a) { return reinterpret_cast<uintptr_t>(q) % a == 0; };
  const int vbytes = 4 * esz;
  const bool a_vec = al(A, vbytes) && (p.lda * esz) % vbytes == 0 && (p.stride_a * esz) % vbytes == 0 &&
                     (p.stride_a2 * esz) % vbytes == 0;
  const bool b_vec = al(B, vbytes) && (p.ldb * esz) % vbytes == 0 && (p.stride_b * esz) % vbytes == 0 &&
                     (p.stride_b2 * esz) % vbytes == 0;
  dim3 grid((unsigned)((p.N + BN - 1) / BN), (unsigned)((p.M + BM - 1) / BM), (unsigned)p.batch);
  if (p.b_layout == DP_B_NK)
    dp::launch_k(sgemm_kernel<TA, TB, true>, grid, kThreads, 0, s, p, static_cast<const TA *>(A),
                                                          static_cast<const TB *>(B), C, bias, res, a_vec, b_vec);
  else
    dp::launch_k(sgemm_kernel<TA, TB, false>, grid, kThreads, 0, s, p, static_cast<const TA *>(A),
                                                           static_cast<const TB *>(B), C, bias, res, a_vec, b_vec);
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

}  // namespace dpk_sgemm

namespace dp {

int launch_gemm_simt(const dp_gemm_params &p, const void *A, const void *B, void *C, const void *bias,
                     const void *res, cudaStream_t s) {
  // TF32 operands that cannot go to the tensor cores run in full fp32 here.
  if ((p.a_dtype == DP_F32 || p.a_dtype == DP_TF32) && (p.b_dtype == DP_F32 || p.b_dtype == DP_TF32))
    return dpk_sgemm::launch_typed<float, float>(p, A, B, C, bias, res, s);
  if (p.a_dtype == DP_BF16 && p.b_dtype == DP_BF16)
    return dpk_sgemm::launch_typed<__nv_bfloat16, __nv_bfloat16>(p, A, B, C, bias, res, s);
  return set_error(DP_ERR_UNSUPPORTED, "gemm: FFMA path takes f32×f32 or bf16×bf16");
}

}  // namespace dp
