// Fused preprocessing region: image load → bilinear resize → fp32 cast →
// (x - mean[c]) / std[c] → layout change → store, in one HBM pass.
//
// Replaces the reference's per-op chain handle_resize (F.interpolate) →
// normalize_kernel → to_dtype_kernel → handle_transpose
// (src/devproc/backend/triton/ops.py:21-53, 320-432; templates/elementwise.py).
//
// Work unit = one output row (image b, output row y).  It needs input rows
// y0 and y0+1 of every channel plane; they are adjacent in memory, so one
// bulk copy (TMA engine, cp.async.bulk) per plane stages them in shared
// memory.  A persistent block keeps STAGES units in flight (mbarrier per
// stage) while its threads compute the current row: thread x produces output
// column x of every channel, so stores are coalesced per channel plane.
//
// Arithmetic follows torch's CPU upsample_bilinear2d (torch 2.11,
// align_corners=False) operation for operation, which makes the result
// bit-identical to F.interpolate on float input:
//   scale = in / out (fp32); src = fma(scale, o + 0.5, -0.5), clamped at 0;
//   i0 = min(floor(src), in-1); l1 = clamp(src - i0, 0, 1); l0 = 1 - l1;
//   i1 = i0 + (i0 < in-1); equal sizes copy (l0 = 1, l1 = 0);
//   row = fma(x[i0], l0, x[i1] * l1); out = fma(row0, h0, row1 * h1).
#include "dp_common.cuh"

namespace dpk_preproc {

constexpr int kStages = 4;
constexpr int kMaxThreads = 256;

struct Coef {
  int i0, i1;
  float l0, l1;
};

__device__ __forceinline__ Coef src_coef(int o, int in_size, int out_size, float scale) {
  Coef c;
  if (in_size == out_size) {
    c.i0 = c.i1 = o;
    c.l0 = 1.0f;
    c.l1 = 0.0f;
    return c;
  }
  float src = __fmaf_rn(scale, (float)o + 0.5f, -0.5f);
  if (src < 0.0f) src = 0.0f;
  int i0 = (int)floorf(src);
  if (i0 > in_size - 1) i0 = in_size - 1;
  float l1 = fminf(fmaxf(__fsub_rn(src, (float)i0), 0.0f), 1.0f);
  c.i0 = i0;
  c.i1 = i0 + (i0 < in_size - 1 ? 1 : 0);
  c.l1 = l1;
  c.l0 = __fsub_rn(1.0f, l1);
  return c;
}

struct Geo {
  int B, H, W, C, OH, OW;
  int planes;          // 1 for NHWC input, C for NCHW
  int row_elems;       // elements of one input row of one plane
  int rows_staged;     // 2, or 1 when H == 1
  int plane_stride_s;  // elements between planes in a smem stage (16-B padded)
  float sy, sx;
  int normalize;
  float mean[4], inv_unused[4], stdv[4];
};

template <typename TIn, bool IN_NCHW>
__device__ __forceinline__ const TIn *plane_src(const TIn *in, const Geo &g, int b, int plane, int y_start) {
  if (IN_NCHW) return in + ((int64_t)(b * g.C + plane) * g.H + y_start) * g.W;
  return in + ((int64_t)b * g.H + y_start) * (int64_t)g.W * g.C;
}

// Computes output row (b, oy) from the staged rows in ``st``.
template <typename TIn, typename TOut, bool IN_NCHW, bool OUT_NCHW>
__device__ __forceinline__ void compute_row(const TIn *st, const Geo &g, int b, int oy, int y_start,
                                            TOut *out, const Coef &cx_first) {
  Coef cy = src_coef(oy, g.H, g.OH, g.sy);
  const int r0 = cy.i0 - y_start, r1 = cy.i1 - y_start;
  for (int ox = threadIdx.x; ox < g.OW; ox += blockDim.x) {
    const Coef cx = (ox == (int)threadIdx.x) ? cx_first : src_coef(ox, g.W, g.OW, g.sx);
#pragma unroll 4
    for (int c = 0; c < g.C; ++c) {
      const TIn *p0, *p1;
      int e0, e1;
      if (IN_NCHW) {
        p0 = st + c * g.plane_stride_s + r0 * g.row_elems;
        p1 = st + c * g.plane_stride_s + r1 * g.row_elems;
        e0 = cx.i0;
        e1 = cx.i1;
      } else {
        p0 = st + r0 * g.row_elems;
        p1 = st + r1 * g.row_elems;
        e0 = cx.i0 * g.C + c;
        e1 = cx.i1 * g.C + c;
      }
      float a = to_f32(p0[e0]), bb = to_f32(p0[e1]);
      float cc = to_f32(p1[e0]), d = to_f32(p1[e1]);
      float row0 = __fmaf_rn(a, cx.l0, __fmul_rn(bb, cx.l1));
      float row1 = __fmaf_rn(cc, cx.l0, __fmul_rn(d, cx.l1));
      float v = __fmaf_rn(row0, cy.l0, __fmul_rn(row1, cy.l1));
      if (g.normalize) v = __fdiv_rn(__fsub_rn(v, g.mean[c]), g.stdv[c]);
      int64_t o;
      if (OUT_NCHW)
        o = (((int64_t)b * g.C + c) * g.OH + oy) * g.OW + ox;
      else
        o = (((int64_t)b * g.OH + oy) * g.OW + ox) * g.C + c;
      out[o] = from_f32<TOut>(v);
    }
  }
}

__device__ __forceinline__ int staged_start(int oy, const Geo &g) {
  if (g.rows_staged == 1) return 0;
  Coef cy = src_coef(oy, g.H, g.OH, g.sy);
  return cy.i0 < g.H - 1 ? cy.i0 : g.H - 2;
}

// TMA path: every plane's staged rows are 16-byte aligned, multiple-of-16
// sized, and rows_staged * row bytes fits one bulk copy.
template <typename TIn, typename TOut, bool IN_NCHW, bool OUT_NCHW>
__global__ void __launch_bounds__(kMaxThreads) preproc_bulk_kernel(Geo g, const TIn *__restrict__ in,
                                                                   TOut *__restrict__ out, int n_units) {
  dp::pdl_trigger();
  dp::pdl_wait();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kStages];
  const int stage_elems = g.planes * g.plane_stride_s;
  TIn *stage0 = reinterpret_cast<TIn *>(smem_raw);
  const uint32_t plane_bytes = (uint32_t)(g.rows_staged * g.row_elems * sizeof(TIn));
  const uint32_t stage_bytes = plane_bytes * g.planes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int k) {  // thread 0 only: stage unit #k of this block
    const int u = blockIdx.x + k * gridDim.x;
    if (u >= n_units) return;
    const int b = u / g.OH, oy = u % g.OH;
    const int ys = staged_start(oy, g);
    const int s = k % kStages;
    mbar_arrive_expect_tx(&bars[s], stage_bytes);
    for (int p = 0; p < g.planes; ++p)
      bulk_g2s(stage0 + s * stage_elems + p * g.plane_stride_s, plane_src<TIn, IN_NCHW>(in, g, b, p, ys),
               plane_bytes, &bars[s]);
  };

  const int my_units = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  if (threadIdx.x == 0)
    for (int k = 0; k < kStages && k < my_units; ++k) issue(k);

  const Coef cx_first = src_coef((int)threadIdx.x < g.OW ? (int)threadIdx.x : 0, g.W, g.OW, g.sx);
  int k = 0;
  for (; k < my_units; ++k) {
    const int s = k % kStages;
    const uint32_t phase = (uint32_t)(k / kStages) & 1u;
    // A thread whose wait gave up still computes (on possibly stale data,
    // with the error word set) so that the block stays in lock-step; the
    // vote below then stops the whole block together.
    const bool ok = mbar_wait_bounded(&bars[s], phase, 100 + s);
    const int u = blockIdx.x + k * gridDim.x;
    const int b = u / g.OH, oy = u % g.OH;
    compute_row<TIn, TOut, IN_NCHW, OUT_NCHW>(stage0 + s * stage_elems, g, b, oy, staged_start(oy, g), out,
                                              cx_first);
    if (!__syncthreads_and(ok)) break;  // also: everyone is done reading stage s
    if (threadIdx.x == 0 && k + kStages < my_units) issue(k + kStages);
  }
  if (k < my_units && threadIdx.x == 0) {
    // Drain: wait (bounded) for every copy this block still has in flight
    // (units k .. k+kStages-1) before its shared memory goes away.
    for (int j = k; j < my_units && j < k + kStages; ++j)
      mbar_wait_bounded(&bars[j % kStages], (uint32_t)(j / kStages) & 1u, 199, 100000000ull);
  }
  __syncthreads();
}

// Plain-load path for sizes or alignments the bulk copy cannot take.
template <typename TIn, typename TOut, bool IN_NCHW, bool OUT_NCHW>
__global__ void __launch_bounds__(kMaxThreads) preproc_plain_kernel(Geo g, const TIn *__restrict__ in,
                                                                    TOut *__restrict__ out, int n_units) {
  dp::pdl_trigger();
  dp::pdl_wait();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  TIn *st = reinterpret_cast<TIn *>(smem_raw);
  const int plane_elems = g.rows_staged * g.row_elems;
  const Coef cx_first = src_coef((int)threadIdx.x < g.OW ? (int)threadIdx.x : 0, g.W, g.OW, g.sx);
  for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
    const int b = u / g.OH, oy = u % g.OH;
    const int ys = staged_start(oy, g);
    for (int p = 0; p < g.planes; ++p) {
      const TIn *src = plane_src<TIn, IN_NCHW>(in, g, b, p, ys);
      for (int i = threadIdx.x; i < plane_elems; i += blockDim.x) st[p * g.plane_stride_s + i] = src[i];
    }
    __syncthreads();
    compute_row<TIn, TOut, IN_NCHW, OUT_NCHW>(st, g, b, oy, ys, out, cx_first);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Fast path: uint8 NHWC, 3 channels, even output width, input width a
// multiple of 16 (so every staged row is 16-byte aligned), planar output.
// Each thread produces two adjacent output columns of one output row for all
// three channels; a block covers R output rows per unit.  Per output element
// the kernel spends ~16 full-rate instructions:
//   * the 6 bytes of an (x0, x0+1) pixel pair come from three 4-byte shared
//     loads plus funnel shifts; byte → float is exact via the 2^23 magic
//     number (byte | 0x4B000000 reinterpreted, minus 2^23) instead of I2F;
//   * the three interpolation FMAs are the generic path's, unchanged;
//   * (v - mean) / std is computed as the correctly rounded quotient with
//     Markstein's FMA correction (P. Markstein, "Computation of elementary
//     functions on the IBM RISC System/6000 processor", IBM J. R&D 34(1),
//     1990): y = RN(1/std) precomputed on the host, q = RN(t·y),
//     r = fma(-q, std, t) (exact), result = RN(q + r·y) — equal to IEEE
//     t / std for these finite, normal operands;
//   * two output columns are packed into one 32-bit (bf16/f16) or 64-bit
//     (f32) store per channel.
constexpr int kFastStages = 2;

struct FastGeo {
  int B, H, W, OH, OW;
  int R, tpr, upi;     // rows per unit, threads per row, units per image
  int split, rps;      // thread groups sharing a unit's rows, rows per group
  int row_bytes;       // W * 3
  int slot_bytes;      // shared bytes per output row: 2 input rows + 16 B slack, 16-B rounded
  float sy, sx;
  int normalize;
  float mean[3], stdv[3], rcp[3];
};


// Window of one output column: the three 4-byte words of the row holding
// pixels x0 and x1 (from the word containing x0's first byte), and how to
// shift them so that pixel x0 starts at byte 0.  ``edge`` marks the clamped
// right edge (x1 == x0).  Three 32-bit shared loads and two funnel shifts per
// pixel pair: no selects, and the 16 bytes of slack after each staged row
// cover the last word.
struct ColWin {
  int ws;
  int sh;
  bool edge;
  float l0, l1;
};

__device__ __forceinline__ ColWin make_win(const Coef &c) {
  ColWin w;
  const int b0 = 3 * c.i0;
  w.ws = b0 & ~3;
  w.sh = 8 * (b0 & 3);
  w.edge = c.i1 == c.i0;
  w.l0 = c.l0;
  w.l1 = c.l1;
  return w;
}

// Bytes of pixels x0 and x0+1 (3 channels each) as a0 = [x0.c0 x0.c1 x0.c2 x1.c0],
// a1 = [x1.c1 x1.c2 . .].
__device__ __forceinline__ void fetch_pair(const uint8_t *row, const ColWin &w, uint32_t &a0, uint32_t &a1) {
  const uint32_t *q = reinterpret_cast<const uint32_t *>(row + w.ws);
  const uint32_t w0 = q[0], w1 = q[1], w2 = q[2];
  a0 = __funnelshift_r(w0, w1, w.sh);
  a1 = __funnelshift_r(w1, w2, w.sh);
}


// Output values of one channel at the thread's two columns, computed as f32x2
// pairs (sm_100 packed FMA/ADD/MUL; each lane rounds exactly like the scalar
// instruction, so the arithmetic is the generic path's, two columns at once).
// Bytes are turned into floats by building the bits of 2^23 + byte with one
// byte permute and subtracting 2^23.
template <int SEL>
__device__ __forceinline__ float magic_bits(uint32_t word) {
  return __int_as_float((int)__byte_perm(word, 0x4B000000u, 0x7440u | (unsigned)SEL));
}

template <int C, bool EDGE>
__device__ __forceinline__ float2 pair_value(uint32_t p0a, uint32_t p0b, uint32_t p1a, uint32_t p1b,  // col 0
                                             uint32_t q0a, uint32_t q0b, uint32_t q1a, uint32_t q1b,  // col 1
                                             float2 L0, float2 L1, float2 H0, float2 H1, const FastGeo &g) {
  const float2 m23 = make_float2(-8388608.0f, -8388608.0f);
  // pixel x0 of both columns, rows 0 and 1
  const float2 A = __fadd2_rn(make_float2(magic_bits<C>(p0a), magic_bits<C>(q0a)), m23);
  const float2 Cc = __fadd2_rn(make_float2(magic_bits<C>(p1a), magic_bits<C>(q1a)), m23);
  // pixel x1: byte C+3 of the pair window (column 1 repeats x0 at the right edge)
  float b0, b1, d0, d1;
  if constexpr (C == 0) {
    b0 = magic_bits<3>(p0a);
    d0 = magic_bits<3>(p1a);
  } else {
    b0 = magic_bits<C - 1>(p0b);
    d0 = magic_bits<C - 1>(p1b);
  }
  if constexpr (EDGE) {
    b1 = magic_bits<C>(q0a);
    d1 = magic_bits<C>(q1a);
  } else if constexpr (C == 0) {
    b1 = magic_bits<3>(q0a);
    d1 = magic_bits<3>(q1a);
  } else {
    b1 = magic_bits<C - 1>(q0b);
    d1 = magic_bits<C - 1>(q1b);
  }
  const float2 B = __fadd2_rn(make_float2(b0, b1), m23);
  const float2 D = __fadd2_rn(make_float2(d0, d1), m23);
  const float2 row0 = __ffma2_rn(A, L0, __fmul2_rn(B, L1));
  const float2 row1 = __ffma2_rn(Cc, L0, __fmul2_rn(D, L1));
  float2 t = __ffma2_rn(row0, H0, __fmul2_rn(row1, H1));
  if (g.normalize) {
    // (t - mean) / std, correctly rounded (Markstein): q = t·y, r = t - q·std, q + r·y.
    t = __fadd2_rn(t, make_float2(-g.mean[C], -g.mean[C]));
    const float2 y = make_float2(g.rcp[C], g.rcp[C]);
    const float2 q = __fmul2_rn(t, y);
    const float2 r = __ffma2_rn(q, make_float2(-g.stdv[C], -g.stdv[C]), t);
    t = __ffma2_rn(r, y, q);
  }
  return t;
}

template <typename TOut>
__device__ __forceinline__ void store_pair(TOut *p, float v0, float v1);
template <>
__device__ __forceinline__ void store_pair<__nv_bfloat16>(__nv_bfloat16 *p, float v0, float v1) {
  *reinterpret_cast<__nv_bfloat162 *>(p) = __floats2bfloat162_rn(v0, v1);
}
template <>
__device__ __forceinline__ void store_pair<__half>(__half *p, float v0, float v1) {
  *reinterpret_cast<__half2 *>(p) = __floats2half2_rn(v0, v1);
}
template <>
__device__ __forceinline__ void store_pair<float>(float *p, float v0, float v1) {
  *reinterpret_cast<float2 *>(p) = make_float2(v0, v1);
}

// Vertical coefficients of every output row, built once per block in shared
// memory: first staged input row, rows of y0/y1 inside the staged pair, weights.
struct RowCoef {
  int ys;
  int r01;  // (y0 - ys) | (y1 - ys) << 8
  float h0, h1;
};

template <typename TOut, bool C1_EDGE>
__device__ __forceinline__ void compute_two_cols(const uint8_t *row0, const uint8_t *row1, const ColWin &c0,
                                                 const ColWin &c1, float h0, float h1, const FastGeo &g,
                                                 TOut *o, int64_t plane) {
  uint32_t p0a, p0b, p1a, p1b, q0a, q0b, q1a, q1b;
  fetch_pair(row0, c0, p0a, p0b);
  fetch_pair(row1, c0, p1a, p1b);
  fetch_pair(row0, c1, q0a, q0b);
  fetch_pair(row1, c1, q1a, q1b);
  const float2 L0 = make_float2(c0.l0, c1.l0), L1 = make_float2(c0.l1, c1.l1);
  const float2 H0 = make_float2(h0, h0), H1 = make_float2(h1, h1);
  float2 v = pair_value<0, C1_EDGE>(p0a, p0b, p1a, p1b, q0a, q0b, q1a, q1b, L0, L1, H0, H1, g);
  store_pair<TOut>(o, v.x, v.y);
  v = pair_value<1, C1_EDGE>(p0a, p0b, p1a, p1b, q0a, q0b, q1a, q1b, L0, L1, H0, H1, g);
  store_pair<TOut>(o + plane, v.x, v.y);
  v = pair_value<2, C1_EDGE>(p0a, p0b, p1a, p1b, q0a, q0b, q1a, q1b, L0, L1, H0, H1, g);
  store_pair<TOut>(o + 2 * plane, v.x, v.y);
}

constexpr int kMaxFastOH = 2048;
constexpr int kFastRowsPerThread = 8;  // output rows a thread computes per unit

// Warp-specialised pipeline: warp 0 lane 0 is the producer (bulk copies into
// kFastStages stages, each guarded by a "full" and an "empty" mbarrier);
// warps 1.. are consumers, one column pair per lane, walking the R output
// rows of each unit.  When the column pairs of a row fill a whole number of
// warps only when doubled (224 output columns: 112 pairs, 3.5 warps), two
// thread groups split each unit's rows (R/2 each), so every consumer lane
// works (7 full warps instead of 4 with 16 idle lanes).  Consumers never wait
// for each other: a warp releases a
// stage with one arrive on its "empty" barrier.  Every wait is bounded; a
// timeout sets the device error word and a shared abort flag, after which
// all warps stop and the producer waits (bounded) for the copies it issued.
template <typename TOut>
__global__ void __launch_bounds__(kMaxThreads + 32) preproc_u8c3_kernel(FastGeo g, const uint8_t *__restrict__ in,
                                                                        TOut *__restrict__ out, int n_units) {
  dp::pdl_trigger();
  dp::pdl_wait();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[kFastStages];
  __shared__ __align__(8) uint64_t empty[kFastStages];
  __shared__ int abort_flag;
  const int stage_bytes = g.R * g.slot_bytes;
  const uint32_t copy_bytes = (uint32_t)(2 * g.row_bytes);
  RowCoef *rows = reinterpret_cast<RowCoef *>(smem_raw + kFastStages * stage_bytes);
  const int n_consumer_warps = (g.split * g.tpr + 31) / 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFastStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], n_consumer_warps);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  for (int oy = threadIdx.x; oy < g.OH; oy += blockDim.x) {
    const Coef cy = src_coef(oy, g.H, g.OH, g.sy);
    RowCoef rc;
    rc.ys = cy.i0 < g.H - 1 ? cy.i0 : g.H - 2;
    rc.r01 = (cy.i0 - rc.ys) | ((cy.i1 - rc.ys) << 8);
    rc.h0 = cy.l0;
    rc.h1 = cy.l1;
    rows[oy] = rc;
  }
  __syncthreads();

  const int my_units = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int k = 0; k < my_units; ++k) {
        const int s = k % kFastStages;
        if (k >= kFastStages &&
            !mbar_wait_bounded(&empty[s], (uint32_t)((k / kFastStages) - 1) & 1u, 130 + s)) {
          atomicExch(&abort_flag, 1);
          break;
        }
        if (*(volatile int *)&abort_flag) break;
        const int u = blockIdx.x + k * gridDim.x;
        const int b = u / g.upi;
        const int oy0 = (u - b * g.upi) * g.R;
        const int nrows = min(g.R, g.OH - oy0);
        mbar_arrive_expect_tx(&full[s], copy_bytes * nrows);
        for (int rr = 0; rr < nrows; ++rr) {
          const uint8_t *src = in + ((int64_t)b * g.H + rows[oy0 + rr].ys) * g.row_bytes;
          bulk_g2s(smem_raw + s * stage_bytes + rr * g.slot_bytes, src, copy_bytes, &full[s]);
        }
        issued = k + 1;
      }
      if (*(volatile int *)&abort_flag) {
        // Wait (bounded) for the copies of the last kFastStages issued units.
        for (int k = issued - kFastStages < 0 ? 0 : issued - kFastStages; k < issued; ++k)
          mbar_wait_bounded(&full[k % kFastStages], (uint32_t)(k / kFastStages) & 1u, 199, 100000000ull);
      }
    }
    return;
  }

  // Consumers: one column pair per lane.
  const int jj = threadIdx.x - 32;
  const int part = jj / g.tpr;
  const int j = jj - part * g.tpr;
  const bool active = part < g.split;
  const int ox = 2 * j;
  const ColWin c0 = make_win(src_coef(active ? ox : 0, g.W, g.OW, g.sx));
  const ColWin c1 = make_win(src_coef(active ? ox + 1 : 0, g.W, g.OW, g.sx));
  const int64_t plane = (int64_t)g.OH * g.OW;
  // Running (image, unit-in-image) of unit blockIdx.x + k * gridDim.x.
  const int step_b = (int)gridDim.x / g.upi, step_u = (int)gridDim.x - step_b * g.upi;
  int cur_b = (int)blockIdx.x / g.upi, cur_u = (int)blockIdx.x - cur_b * g.upi;
  for (int k = 0; k < my_units; ++k) {
    const int s = k % kFastStages;
    if (!mbar_wait_bounded(&full[s], (uint32_t)(k / kFastStages) & 1u, 120 + s)) atomicExch(&abort_flag, 1);
    if (__any_sync(0xffffffffu, *(volatile int *)&abort_flag)) break;
    const int oy0 = cur_u * g.R;
    if (active) {
      const int nrows = min(g.R, g.OH - oy0);
      const int r_lo = part * g.rps;
      const int r_hi = min(r_lo + g.rps, nrows);
      const uint8_t *stage = smem_raw + s * stage_bytes;
      TOut *o = out + ((int64_t)cur_b * 3 * g.OH + oy0 + r_lo) * g.OW + ox;
#pragma unroll 2
      for (int rr = r_lo; rr < r_hi; ++rr) {
        const RowCoef rc = rows[oy0 + rr];
        const uint8_t *base = stage + rr * g.slot_bytes;
        const uint8_t *row0 = base + (rc.r01 & 0xff) * g.row_bytes;
        const uint8_t *row1 = base + (rc.r01 >> 8) * g.row_bytes;
        // With in_w > out_w only the last output column can sit on the
        // clamped right edge, so the first column of a pair never does.
        if (!c1.edge)
          compute_two_cols<TOut, false>(row0, row1, c0, c1, rc.h0, rc.h1, g, o, plane);
        else
          compute_two_cols<TOut, true>(row0, row1, c0, c1, rc.h0, rc.h1, g, o, plane);
        o += g.OW;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    cur_u += step_u;
    cur_b += step_b;
    if (cur_u >= g.upi) {
      cur_u -= g.upi;
      ++cur_b;
    }
  }
}

template <typename TOut>
int launch_fast(const dp_preproc_params &p, const void *in, void *out, cudaStream_t s) {
  FastGeo g;
  g.B = p.batch;
  g.H = p.in_h;
  g.W = p.in_w;
  g.OH = p.out_h;
  g.OW = p.out_w;
  g.tpr = p.out_w / 2;
  g.R = kFastRowsPerThread < g.OH ? kFastRowsPerThread : g.OH;
  g.upi = (g.OH + g.R - 1) / g.R;
  g.row_bytes = 3 * p.in_w;
  g.slot_bytes = ((2 * g.row_bytes + 16) + 15) / 16 * 16;
  g.sy = (float)p.in_h / (float)p.out_h;
  g.sx = (float)p.in_w / (float)p.out_w;
  g.normalize = p.normalize;
  for (int c = 0; c < 3; ++c) {
    g.mean[c] = p.normalize ? p.mean[c] : 0.0f;
    g.stdv[c] = p.normalize ? p.stdv[c] : 1.0f;
    g.rcp[c] = 1.0f / g.stdv[c];
  }
  g.split = (g.tpr % 32 != 0 && (2 * g.tpr) % 32 == 0 && g.R % 2 == 0 && 2 * g.tpr <= kMaxThreads) ? 2 : 1;
  g.rps = g.R / g.split;
  const int threads = 32 + ((g.split * g.tpr + 31) / 32) * 32;
  const size_t smem = (size_t)kFastStages * g.R * g.slot_bytes + (size_t)g.OH * sizeof(RowCoef);
  const int n_units = g.B * g.upi;
  auto kern = preproc_u8c3_kernel<TOut>;
  int per_sm = 0;
  int st = dp::kernel_blocks_per_sm((const void *)kern, threads, smem, true, &per_sm);
  if (st != DP_OK) return st;
  int grid = dp::num_sms() * per_sm;
  if (grid > n_units) grid = n_units;
  dp::launch_k(kern, grid, threads, smem, s, g, static_cast<const uint8_t *>(in), static_cast<TOut *>(out), n_units);
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

template <typename TIn, typename TOut, bool IN_NCHW, bool OUT_NCHW>
int launch_typed(const Geo &g, const void *in, void *out, cudaStream_t s) {
  const int n_units = g.B * g.OH;
  const int threads = g.OW >= kMaxThreads ? kMaxThreads : ((g.OW + 31) / 32) * 32;
  const size_t stage_bytes = (size_t)g.planes * g.plane_stride_s * sizeof(TIn);
  const uintptr_t base = reinterpret_cast<uintptr_t>(in);
  const size_t plane_bytes = (size_t)g.rows_staged * g.row_elems * sizeof(TIn);
  const size_t row_bytes = (size_t)g.row_elems * sizeof(TIn);
  // Every copy source is base + k * row_bytes (k integer), so 16-B alignment
  // of base and of row_bytes makes every copy aligned.
  const bool bulk = (base % 16 == 0) && (row_bytes % 16 == 0) && (plane_bytes % 16 == 0) &&
                    (plane_bytes < (1u << 20)) && (stage_bytes * kStages <= 200 * 1024);
  const int sms = dp::num_sms();
  if (bulk) {
    auto kern = preproc_bulk_kernel<TIn, TOut, IN_NCHW, OUT_NCHW>;
    const size_t smem = stage_bytes * kStages;
    int per_sm = 0;
    int st = dp::kernel_blocks_per_sm((const void *)kern, threads, smem, false, &per_sm);
    if (st != DP_OK) return st;
    int grid = sms * per_sm;
    if (grid > n_units) grid = n_units;
    dp::launch_k(kern, grid, threads, smem, s, g, static_cast<const TIn *>(in), static_cast<TOut *>(out), n_units);
  } else {
    auto kern = preproc_plain_kernel<TIn, TOut, IN_NCHW, OUT_NCHW>;
    const size_t smem = stage_bytes;
    DP_REQUIRE(smem <= 200 * 1024, DP_ERR_UNSUPPORTED, "preproc: input rows too wide for shared memory");
    int per_sm = 0;
    int st = dp::kernel_blocks_per_sm((const void *)kern, threads, smem, false, &per_sm);
    if (st != DP_OK) return st;
    int grid = sms * per_sm;
    if (grid > n_units) grid = n_units;
    dp::launch_k(kern, grid, threads, smem, s, g, static_cast<const TIn *>(in), static_cast<TOut *>(out), n_units);
  }
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

template <typename TIn, typename TOut>
int launch_layouts(const Geo &g, bool in_nchw, bool out_nchw, const void *in, void *out, cudaStream_t s) {
  if (in_nchw) {
    return out_nchw ? launch_typed<TIn, TOut, true, true>(g, in, out, s)
                    : launch_typed<TIn, TOut, true, false>(g, in, out, s);
  }
  return out_nchw ? launch_typed<TIn, TOut, false, true>(g, in, out, s)
                  : launch_typed<TIn, TOut, false, false>(g, in, out, s);
}

template <typename TIn>
int launch_out(const Geo &g, int out_dtype, bool in_nchw, bool out_nchw, const void *in, void *out,
               cudaStream_t s) {
  switch (out_dtype) {
    case DP_F32: return launch_layouts<TIn, float>(g, in_nchw, out_nchw, in, out, s);
    case DP_BF16: return launch_layouts<TIn, __nv_bfloat16>(g, in_nchw, out_nchw, in, out, s);
    case DP_F16: return launch_layouts<TIn, __half>(g, in_nchw, out_nchw, in, out, s);
    default: return dp::set_error(DP_ERR_UNSUPPORTED, "preproc: output dtype must be f32, bf16 or f16");
  }
}

}  // namespace dpk_preproc

using namespace dpk_preproc;

namespace dp {

int launch_preproc(const dp_preproc_params &p, const void *in, void *out, cudaStream_t s) {
  DP_REQUIRE(in && out, DP_ERR_ARG, "preproc: null pointer");
  DP_REQUIRE(p.batch > 0 && p.in_h > 0 && p.in_w > 0 && p.out_h > 0 && p.out_w > 0, DP_ERR_SHAPE,
             "preproc: sizes must be positive");
  DP_REQUIRE(p.channels >= 1 && p.channels <= 4, DP_ERR_UNSUPPORTED, "preproc: 1 to 4 channels");
  DP_REQUIRE((int64_t)p.batch * p.out_h < (1ll << 31), DP_ERR_UNSUPPORTED, "preproc: too many output rows");
  DP_REQUIRE(p.in_layout == DP_LAYOUT_NHWC || p.in_layout == DP_LAYOUT_NCHW, DP_ERR_ARG, "preproc: in_layout");
  DP_REQUIRE(p.out_layout == DP_LAYOUT_NHWC || p.out_layout == DP_LAYOUT_NCHW, DP_ERR_ARG, "preproc: out_layout");
  Geo g;
  g.B = p.batch;
  g.H = p.in_h;
  g.W = p.in_w;
  g.C = p.channels;
  g.OH = p.out_h;
  g.OW = p.out_w;
  const bool in_nchw = p.in_layout == DP_LAYOUT_NCHW;
  g.planes = in_nchw ? p.channels : 1;
  g.row_elems = in_nchw ? p.in_w : p.in_w * p.channels;
  g.rows_staged = p.in_h >= 2 ? 2 : 1;
  const int eb = dtype_bytes(p.in_dtype);
  DP_REQUIRE(eb > 0, DP_ERR_ARG, "preproc: bad input dtype");
  // Pad each staged plane to 16 bytes so every bulk destination is aligned.
  const int plane_elems = g.rows_staged * g.row_elems;
  const int pad = 16 / eb;
  g.plane_stride_s = ((plane_elems + pad - 1) / pad) * pad;
  g.sy = (float)p.in_h / (float)p.out_h;
  g.sx = (float)p.in_w / (float)p.out_w;
  g.normalize = p.normalize;
  for (int c = 0; c < 4; ++c) {
    g.mean[c] = p.normalize ? p.mean[c] : 0.0f;
    g.stdv[c] = p.normalize ? p.stdv[c] : 1.0f;
    g.inv_unused[c] = 0.0f;
    if (p.normalize && c < p.channels)
      DP_REQUIRE(p.stdv[c] != 0.0f, DP_ERR_ARG, "preproc: std must be non-zero");
  }
  const bool out_nchw = p.out_layout == DP_LAYOUT_NCHW;
  const bool fast = p.in_dtype == DP_U8 && !in_nchw && out_nchw && p.channels == 3 && p.in_w % 16 == 0 &&
                    p.out_w % 2 == 0 && p.in_h >= 2 && reinterpret_cast<uintptr_t>(in) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(out) % 8 == 0 && 2 * 3 * p.in_w + 16 <= 12 * 1024 &&
                    p.out_w / 2 <= kMaxThreads && p.out_h <= kMaxFastOH && p.in_w > p.out_w;
  if (fast) {
    switch (p.out_dtype) {
      case DP_BF16: return launch_fast<__nv_bfloat16>(p, in, out, s);
      case DP_F16: return launch_fast<__half>(p, in, out, s);
      case DP_F32: return launch_fast<float>(p, in, out, s);
      default: break;
    }
  }
  switch (p.in_dtype) {
    case DP_U8: return launch_out<uint8_t>(g, p.out_dtype, in_nchw, out_nchw, in, out, s);
    case DP_F32: return launch_out<float>(g, p.out_dtype, in_nchw, out_nchw, in, out, s);
    case DP_BF16: return launch_out<__nv_bfloat16>(g, p.out_dtype, in_nchw, out_nchw, in, out, s);
    case DP_F16: return launch_out<__half>(g, p.out_dtype, in_nchw, out_nchw, in, out, s);
    default: return set_error(DP_ERR_UNSUPPORTED, "preproc: input dtype must be u8, f32, bf16 or f16");
  }
}

}  // namespace dp

extern "C" int dp_preproc(const dp_preproc_params *p, const void *in, void *out, void *stream) {
  if (!p) return dp::set_error(DP_ERR_ARG, "dp_preproc: null params");
  return dp::launch_preproc(*p, in, out, dp::as_stream(stream));
}
