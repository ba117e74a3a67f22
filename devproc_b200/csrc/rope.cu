// Rotary position embedding (rotate-half form) as one memory-bound pass.
//
// The reference has no rotary embedding: its FX converter turned the
// textbook slice / neg / cat / mul / add chain into same-shape placeholder
// ops (src/devproc/ir/fx_converter.py:443-448).  Here the ``rope`` IR op is
// one kernel: each thread owns VEC = 16 / sizeof(T) consecutive columns i of
// the first half of one row and the matching columns i + dim/2, so it reads
// both halves of x and the table entries it needs with 16-byte loads and
// writes both output halves with 16-byte stores.  x is read once and the
// output written once (4·dim bytes per 16-bit row); the tables are small and
// stay in L2.  The arithmetic is the torch-level definition's, product by
// product in fp32 without FMA contraction:
//   out1 = x1·c1 − x2·s1,  out2 = x2·c2 + x1·s2,
// rounded once to the output type.
//
// Work item u = ((b·heads + h)·rows + r)·jn + j, where jn = dim / (2·VEC);
// its coordinates come from three FastDiv divisions (items < 2^31).
#include "dp_common.cuh"

namespace dpk_rope {

constexpr int kThreads = 256;

struct RopeGeo {
  int64_t x_sb, x_sh, x_sr;
  int64_t o_sb, o_sh, o_sr;
  int64_t t_sb, t_sh, t_sr;
  int64_t half;    // dim / 2
  int64_t t_half;  // column offset of the second table half (0 for half tables)
  uint32_t items;
  FastDiv jn, rows, heads;
};

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// N elements of T at p (aligned to min(16, N·sizeof(T)) bytes) as floats.
template <typename T, int N>
__device__ __forceinline__ void load_vec(const T *p, float (&v)[N]) {
  constexpr int kBytes = N * (int)sizeof(T);
  static_assert(kBytes % 8 == 0, "vector of at least 8 bytes");
  T tmp[N];
  if constexpr (kBytes % 16 == 0) {
#pragma unroll
    for (int w = 0; w < kBytes / 16; ++w)
      reinterpret_cast<uint4 *>(tmp)[w] = __ldg(reinterpret_cast<const uint4 *>(p) + w);
  } else {
    reinterpret_cast<uint2 *>(tmp)[0] = __ldg(reinterpret_cast<const uint2 *>(p));
  }
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = to_f32(tmp[i]);
}

template <typename T, int N>
__device__ __forceinline__ void store_vec(T *p, const float (&v)[N]) {
  static_assert(N * sizeof(T) == 16, "16-byte stores");
  T tmp[N];
#pragma unroll
  for (int i = 0; i < N; ++i) tmp[i] = from_f32<T>(v[i]);
  *reinterpret_cast<uint4 *>(p) = *reinterpret_cast<const uint4 *>(tmp);
}

template <typename TX, typename TT>
__global__ void __launch_bounds__(kThreads) rope_kernel(RopeGeo g, const TX *__restrict__ x,
                                                        const TT *__restrict__ cosv, const TT *__restrict__ sinv,
                                                        TX *__restrict__ out) {
  dp::pdl_trigger();
  dp::pdl_wait();
  constexpr int VEC = 16 / (int)sizeof(TX);
  for (uint32_t u = blockIdx.x * (uint32_t)kThreads + threadIdx.x; u < g.items;
       u += gridDim.x * (uint32_t)kThreads) {
    const uint32_t row = fdiv(u, g.jn);
    const uint32_t j = u - row * g.jn.d;
    const uint32_t bh = fdiv(row, g.rows);
    const uint32_t r = row - bh * g.rows.d;
    const uint32_t b = fdiv(bh, g.heads);
    const uint32_t h = bh - b * g.heads.d;
    const int64_t col = (int64_t)j * VEC;
    const TX *xr = x + b * g.x_sb + h * g.x_sh + r * g.x_sr + col;
    const int64_t t = b * g.t_sb + h * g.t_sh + r * g.t_sr + col;
    float x1[VEC], x2[VEC], c1[VEC], s1[VEC], c2[VEC], s2[VEC];
    load_vec<TX, VEC>(xr, x1);
    load_vec<TX, VEC>(xr + g.half, x2);
    load_vec<TT, VEC>(cosv + t, c1);
    load_vec<TT, VEC>(sinv + t, s1);
    load_vec<TT, VEC>(cosv + t + g.t_half, c2);
    load_vec<TT, VEC>(sinv + t + g.t_half, s2);
    float o1[VEC], o2[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      o1[i] = __fsub_rn(__fmul_rn(x1[i], c1[i]), __fmul_rn(x2[i], s1[i]));
      o2[i] = __fadd_rn(__fmul_rn(x2[i], c2[i]), __fmul_rn(x1[i], s2[i]));
    }
    TX *orow = out + b * g.o_sb + h * g.o_sh + r * g.o_sr + col;
    store_vec<TX, VEC>(orow, o1);
    store_vec<TX, VEC>(orow + g.half, o2);
  }
}

template <typename TX, typename TT>
int launch_typed(const RopeGeo &g, const void *x, const void *c, const void *s, void *o, cudaStream_t st) {
  int64_t blocks = ((int64_t)g.items + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)dp::num_sms() * (2048 / kThreads) * 4;
  if (blocks > cap) blocks = cap;
  dp::launch_k(rope_kernel<TX, TT>, (unsigned)blocks, kThreads, 0, st, g, static_cast<const TX *>(x),
                                                              static_cast<const TT *>(c),
                                                              static_cast<const TT *>(s), static_cast<TX *>(o));
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

template <typename TX>
int launch_tables(const RopeGeo &g, int t_dtype, const void *x, const void *c, const void *s, void *o,
                  cudaStream_t st) {
  switch (t_dtype) {
    case DP_BF16: return launch_typed<TX, __nv_bfloat16>(g, x, c, s, o, st);
    case DP_F16: return launch_typed<TX, __half>(g, x, c, s, o, st);
    case DP_F32: return launch_typed<TX, float>(g, x, c, s, o, st);
    default: return dp::set_error(DP_ERR_UNSUPPORTED, "rope: table dtype must be bf16, f16 or f32");
  }
}

}  // namespace dpk_rope

namespace dp {

int launch_rope(const dp_rope_params &p, const void *x, const void *cosv, const void *sinv, void *out,
                cudaStream_t s) {
  DP_REQUIRE(x && cosv && sinv && out, DP_ERR_ARG, "rope: null pointer");
  DP_REQUIRE(p.batch > 0 && p.heads > 0 && p.rows > 0 && p.dim > 0, DP_ERR_SHAPE,
             "rope: sizes must be positive");
  DP_REQUIRE(p.x_dtype == DP_BF16 || p.x_dtype == DP_F16 || p.x_dtype == DP_F32, DP_ERR_UNSUPPORTED,
             "rope: x dtype must be bf16, f16 or f32");
  DP_REQUIRE(p.t_dtype == DP_BF16 || p.t_dtype == DP_F16 || p.t_dtype == DP_F32, DP_ERR_UNSUPPORTED,
             "rope: table dtype must be bf16, f16 or f32");
  const int xb = dtype_bytes(p.x_dtype), tb = dtype_bytes(p.t_dtype);
  const int64_t vec = 16 / xb;
  DP_REQUIRE(p.dim % (2 * vec) == 0, DP_ERR_UNSUPPORTED,
             "rope: dim/2 must be a multiple of " + std::to_string(vec));
  for (int64_t st : {p.x_sb, p.x_sh, p.x_sr, p.o_sb, p.o_sh, p.o_sr})
    DP_REQUIRE(st % vec == 0, DP_ERR_UNSUPPORTED, "rope: x / out strides must be multiples of 16 bytes");
  // a table vector is vec elements of the table type: 8, 16 or 32 bytes
  const int64_t t_align = vec * tb >= 16 ? 16 / tb : vec;
  for (int64_t st : {p.t_sb, p.t_sh, p.t_sr})
    DP_REQUIRE(st >= 0 && st % t_align == 0, DP_ERR_UNSUPPORTED, "rope: table strides not vector-aligned");
  for (const void *q : {x, (const void *)out, cosv, sinv})
    DP_REQUIRE(reinterpret_cast<uintptr_t>(q) % 16 == 0, DP_ERR_UNSUPPORTED,
               "rope: bases must be 16-byte aligned");
  DP_REQUIRE(x != out, DP_ERR_ARG, "rope: out must not overlap x");
  const int64_t jn = p.dim / 2 / vec;
  const int64_t items = p.batch * p.heads * p.rows * jn;
  DP_REQUIRE(items < (1ll << 31), DP_ERR_UNSUPPORTED, "rope: more than 2^31 work items");
  dpk_rope::RopeGeo g;
  g.x_sb = p.x_sb; g.x_sh = p.x_sh; g.x_sr = p.x_sr;
  g.o_sb = p.o_sb; g.o_sh = p.o_sh; g.o_sr = p.o_sr;
  g.t_sb = p.t_sb; g.t_sh = p.t_sh; g.t_sr = p.t_sr;
  g.half = p.dim / 2;
  g.t_half = p.half_table ? 0 : p.dim / 2;
  g.items = (uint32_t)items;
  g.jn = make_fastdiv((uint32_t)jn);
  g.rows = make_fastdiv((uint32_t)p.rows);
  g.heads = make_fastdiv((uint32_t)p.heads);
  switch (p.x_dtype) {
    case DP_BF16: return dpk_rope::launch_tables<__nv_bfloat16>(g, p.t_dtype, x, cosv, sinv, out, s);
    case DP_F16: return dpk_rope::launch_tables<__half>(g, p.t_dtype, x, cosv, sinv, out, s);
    default: return dpk_rope::launch_tables<float>(g, p.t_dtype, x, cosv, sinv, out, s);
  }
}

}  // namespace dp

extern "C" int dp_rope(const dp_rope_params *p, const void *x, const void *cosv, const void *sinv, void *out,
                       void *stream) {
  if (!p) return dp::set_error(DP_ERR_ARG, "dp_rope: null params");
  return dp::launch_rope(*p, x, cosv, sinv, out, dp::as_stream(stream));
}
