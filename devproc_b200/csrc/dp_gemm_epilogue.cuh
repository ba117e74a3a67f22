// GEMM epilogue shared by the FFMA and tcgen05 GEMMs:
//   v = acc (+ bias[n]) → activation → (+ or × residual[m, n]) → cast → C[m, n].
#pragma once

#include "dp_common.cuh"

namespace dp {

__device__ __forceinline__ float act_gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }
__device__ __forceinline__ float act_gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
}

struct Epilogue {
  const dp_gemm_params &p;
  void *C;
  const void *bias;
  const void *res;
  int64_t c_off, r_off;

  __device__ __forceinline__ Epilogue(const dp_gemm_params &p_, void *C_, const void *bias_, const void *res_,
                                      int64_t batch)
      : p(p_), C(C_), bias(bias_), res(res_) {
    const int64_t b2 = p_.batch2 > 1 ? p_.batch2 : 1;
    const int64_t zo = batch / b2, zi = batch - zo * b2;
    c_off = zo * p_.stride_c + zi * p_.stride_c2;
    r_off = zo * p_.stride_r + zi * p_.stride_r2;
  }

  __device__ __forceinline__ float apply(int64_t m, int64_t n, float v) const {
    if (p.alpha != 0.0f) v *= p.alpha;
    if (p.epilogue & DP_EPI_BIAS) v += load_as_f32(bias, n, p.bias_dtype);
    if (p.epilogue & DP_EPI_RELU) v = v > 0.0f ? v : (isnan(v) ? v : 0.0f);
    if (p.epilogue & DP_EPI_GELU_ERF) v = act_gelu_erf(v);
    if (p.epilogue & DP_EPI_GELU_TANH) v = act_gelu_tanh(v);
    if (p.epilogue & DP_EPI_SILU) v = v / (1.0f + expf(-v));
    if (p.epilogue & DP_EPI_RESIDUAL) v += load_as_f32(res, r_off + m * p.ldr + n, p.r_dtype);
    if (p.epilogue & DP_EPI_MUL) v *= load_as_f32(res, r_off + m * p.ldr + n, p.r_dtype);
    return v;
  }

  // Four consecutive columns n .. n+3 of row m (each bounds-checked).
  __device__ __forceinline__ void store4(int64_t m, int64_t n, float v0, float v1, float v2, float v3) const {
    float v[4] = {v0, v1, v2, v3};
    const int64_t base = c_off + m * p.ldc + n;
    if (p.epilogue & DP_EPI_TF32SPLIT) {  // [hi | hi | lo] blocks N columns apart (fp32 C)
      float *c = static_cast<float *>(C) + base;
      float hi[4], lo[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x = n + j < p.N ? apply(m, n + j, v[j]) : 0.0f;
        hi[j] = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
        lo[j] = x - hi[j];
      }
      if (n + 3 < p.N && (base & 3) == 0 && (p.N & 3) == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0) {
        const float4 h4 = make_float4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<float4 *>(c) = h4;
        *reinterpret_cast<float4 *>(c + p.N) = h4;
        *reinterpret_cast<float4 *>(c + 2 * p.N) = make_float4(lo[0], lo[1], lo[2], lo[3]);
        return;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (n + j >= p.N) break;
        c[j] = hi[j];
        c[p.N + j] = hi[j];
        c[2 * p.N + j] = lo[j];
      }
      return;
    }
    if (n + 3 < p.N && p.c_dtype == DP_F32 && (base & 3) == 0 &&
        (reinterpret_cast<uintptr_t>(C) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = apply(m, n + j, v[j]);
      *reinterpret_cast<float4 *>(static_cast<float *>(C) + base) = make_float4(v[0], v[1], v[2], v[3]);
      return;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (n + j < p.N) store_from_f32(C, base + j, p.c_dtype, apply(m, n + j, v[j]));
  }
};

int launch_gemm_simt(const dp_gemm_params &p, const void *A, const void *B, void *C, const void *bias,
                     const void *res, cudaStream_t s);
// sk_workspace (optional): stream-K workspace of sk_bytes; the tile-past-the-
// last-wave split is used only when the cost model picks it and it fits.
int launch_gemm_tc(const dp_gemm_params &p, const void *A, const void *B, void *C, const void *bias,
                   const void *res, cudaStream_t s, void *sk_workspace = nullptr, int64_t sk_bytes = 0);
int64_t gemm_streamk_workspace_bound(const dp_gemm_params &p);

}  // namespace dp
