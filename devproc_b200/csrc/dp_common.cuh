// Shared device/host helpers of the DevProc B200 kernels: status plumbing,
// element conversions, the device error word and bounded mbarrier waits.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>

#include "devproc_b200.h"

// ---------------------------------------------------------------- host side
namespace dp {

// Records the calling thread's last error text; returns ``code``.
int set_error(int code, const std::string &msg);
int cuda_status(cudaError_t e, const char *what);
int num_sms();  // SM count of the current device (cached per device)
// Resident blocks per SM of kernel ``func`` at (threads, smem) on the current
// device.  The first call per (device, kernel, threads, smem) grants the
// dynamic shared-memory opt-in (and, with ``max_carveout``, prefers the
// largest shared-memory carveout) and queries the occupancy; later calls are
// a cache lookup, so launchers make no attribute or occupancy call per launch.
int kernel_blocks_per_sm(const void *func, int threads, size_t smem, bool max_carveout, int *per_sm);

#define DP_CHECK_CUDA(expr)                                   \
  do {                                                        \
    cudaError_t _e = (expr);                                  \
    if (_e != cudaSuccess) return ::dp::cuda_status(_e, #expr); \
  } while (0)

#define DP_REQUIRE(cond, code, msg)                 \
  do {                                              \
    if (!(cond)) return ::dp::set_error((code), (msg)); \
  } while (0)

// Programmatic dependent launch.  Every kernel of this library is launched
// with launch_k, which lets its grid start while the kernel before it on the
// stream is still finishing, and every kernel calls pdl_wait() before its
// first global-memory access (read or write): griddepcontrol.wait returns once
// the previous grid has completed and its writes are visible, so stream order
// holds.  pdl_trigger() at kernel entry lets the next grid launch as soon as
// every CTA of this one has started; its CTAs then take SMs as this grid's
// CTAs exit, instead of after the last one.  Both are no-ops for a grid
// launched without the attribute.  Build switch: DP_PDL=0 launches plainly.
#ifndef DP_PDL
#define DP_PDL 1
#endif
__device__ __forceinline__ void pdl_wait() {
#if DP_PDL
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}
__device__ __forceinline__ void pdl_trigger() {
#if DP_PDL
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = DP_PDL ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

inline int dtype_bytes(int dt) {
  switch (dt) {
    case DP_U8: case DP_I8: case DP_BOOL: return 1;
    case DP_I16: case DP_F16: case DP_BF16: return 2;
    case DP_I32: case DP_F32: case DP_TF32: return 4;
    case DP_I64: case DP_F64: return 8;
    default: return 0;
  }
}

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// Internal launchers shared by the direct entry points and the program runner.
int launch_preproc(const dp_preproc_params &p, const void *in, void *out, cudaStream_t s);
int launch_rowreduce(const dp_rowreduce_params &p, const void *in, const void *w,
                     const void *b, void *out, cudaStream_t s);
// sk_workspace / sk_bytes: optional stream-K workspace (dp_gemm_streamk).
int launch_gemm(const dp_gemm_params &p, const void *A, const void *B, void *C,
                const void *bias, const void *res, cudaStream_t s, void *sk_workspace = nullptr,
                int64_t sk_bytes = 0);
int launch_gemm_streamk(const dp_streamk_params &p, const void *A, const void *B, void *C, const void *bias,
                        const void *res, void *workspace, cudaStream_t s);
int launch_region(const dp_region_desc &d, const void *const *ops, cudaStream_t s);
int launch_attention(const dp_attention_params &p, const void *q, const void *k, const void *v, void *o,
                     cudaStream_t s);
int launch_embedding(const dp_embedding_params &p, const void *ids, const void *w,
                     void *out, cudaStream_t s);
int launch_rope(const dp_rope_params &p, const void *x, const void *cos, const void *sin, void *out,
                cudaStream_t s);
int launch_splitk_reduce(const dp_splitk_params &p, const void *ws, void *C, const void *bias, const void *res,
                         cudaStream_t s);
int launch_argmax_keys(const dp_argmax_keys_params &p, void *keys, void *out, cudaStream_t s);

}  // namespace dp

// Division by a run-time invariant d with one multiply-high, add and shift
// (Granlund & Montgomery, "Division by invariant integers using
// multiplication", 1994): q = (umulhi(n, m) + n) >> s with s = ceil(log2 d),
// m = floor(2^32 (2^s - d) / d) + 1, exact for n < 2^31.
struct FastDiv {
  uint32_t d, m, s;
};

inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t s = 0;
  while ((1ull << s) < d) ++s;
  return FastDiv{d, (uint32_t)((((1ull << 32) * ((1ull << s) - d)) / d) + 1), s};
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f) {
  return (__umulhi(n, f.m) + n) >> f.s;
}

// -------------------------------------------------------------- device side
// Device error word: first failure wins (code, info); read and cleared by
// dp_device_error().  The winning code is also stored to a pinned, mapped
// host word (g_dp_err_host, set up by dp_device_init), so the host can see
// after a stream synchronisation that something failed without a CUDA call
// (dp_device_error_pending).  Defined once in dp_api.cu.
extern __device__ unsigned int g_dp_err_code;
extern __device__ long long g_dp_err_info;
extern __device__ int *g_dp_err_host;
// Wall-time limit of the waits that take the device-wide limit (2 s unless
// dp_set_wait_limit changed it), and the failure-detection switch that makes
// the staged row kernel arm its barriers without issuing the copies.
extern __device__ unsigned long long g_dp_wait_limit_ns;
extern __device__ unsigned int g_dp_withhold_copies;

__device__ __forceinline__ void dp_report(unsigned code, long long info) {
  if (atomicCAS(&g_dp_err_code, 0u, code) == 0u) {
    g_dp_err_info = info;
    int *h = g_dp_err_host;
    if (h) *reinterpret_cast<volatile int *>(h) = (int)code;
  }
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<uint8_t>(uint8_t v) { return (float)v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Generic typed load/store by runtime dtype code (used by the region VM).
__device__ __forceinline__ float load_as_f32(const void *p, int64_t i, int dt) {
  switch (dt) {
    case DP_U8: return (float)((const uint8_t *)p)[i];
    case DP_I8: return (float)((const int8_t *)p)[i];
    case DP_BOOL: return ((const uint8_t *)p)[i] ? 1.0f : 0.0f;
    case DP_I16: return (float)((const int16_t *)p)[i];
    case DP_I32: return (float)((const int32_t *)p)[i];
    case DP_I64: return (float)((const long long *)p)[i];
    case DP_F16: return __half2float(((const __half *)p)[i]);
    case DP_BF16: return __bfloat162float(((const __nv_bfloat16 *)p)[i]);
    case DP_F64: return (float)((const double *)p)[i];
    default: return ((const float *)p)[i];
  }
}

// Float → integer conversions follow C / torch: truncate toward zero
// (saturating at the type's range, NaN → 0); bool is (v != 0).
__device__ __forceinline__ void store_from_f32(void *p, int64_t i, int dt, float v) {
  switch (dt) {
    case DP_U8: ((uint8_t *)p)[i] = (uint8_t)__float2int_rz(fminf(fmaxf(v, 0.f), 255.f)); break;
    case DP_I8: ((int8_t *)p)[i] = (int8_t)__float2int_rz(fminf(fmaxf(v, -128.f), 127.f)); break;
    case DP_BOOL: ((uint8_t *)p)[i] = (v != 0.0f) ? 1 : 0; break;
    case DP_I16: ((int16_t *)p)[i] = (int16_t)__float2int_rz(fminf(fmaxf(v, -32768.f), 32767.f)); break;
    case DP_I32: ((int32_t *)p)[i] = __float2int_rz(v); break;
    case DP_I64: ((long long *)p)[i] = __float2ll_rz(v); break;
    case DP_F16: ((__half *)p)[i] = __float2half_rn(v); break;
    case DP_BF16: ((__nv_bfloat16 *)p)[i] = __float2bfloat16_rn(v); break;
    case DP_F64: ((double *)p)[i] = (double)v; break;
    default: ((float *)p)[i] = v; break;
  }
}

// ---------------------------------------------------------- mbarrier / TMA
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait may suspend the thread until the phase completes or a time hint
// passes; DP_MBAR_HINT selects the hint form (build switch for tuning).
#ifndef DP_MBAR_HINT
#define DP_MBAR_HINT ", 100000"
#endif
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2" DP_MBAR_HINT ";\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Acquire at cluster scope: for barriers that other CTAs of the cluster arrive on.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2" DP_MBAR_HINT ";\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits at most ``timeout_ns`` of wall time (%globaltimer); false on timeout.
template <bool kClusterScope = false>
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t phase, uint64_t timeout_ns) {
  auto probe = [&]() { return kClusterScope ? mbar_try_wait_cluster(bar, phase) : mbar_try_wait(bar, phase); };
  if (probe()) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!probe())
    if (globaltimer_ns() - t0 > timeout_ns) return false;
  return true;
}

// Bounded wait: gives up once ``timeout_ns`` of wall time has passed (0 =
// the device-wide limit, g_dp_wait_limit_ns, read only when the first probe
// fails), records DP_DEVERR_TIMEOUT with ``site`` and returns false.  No wait
// in this library can spin forever.  Waits that drain copies still in flight
// before a CTA exits pass their own fixed limit, so a short device-wide limit
// never lets a CTA leave while a copy can still land in its shared memory.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase, int site,
                                                  uint64_t timeout_ns = 0) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t limit = timeout_ns ? timeout_ns : *reinterpret_cast<volatile unsigned long long *>(&g_dp_wait_limit_ns);
  if (mbar_wait_for(bar, phase, limit)) return true;
  dp_report(DP_DEVERR_TIMEOUT, site);
  return false;
}

// 1-D bulk copy global → shared (TMA engine), completion on ``bar``.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
