// bf16 GEMM on the 5th-generation tensor cores: tcgen05.mma with the fp32
// accumulator in tensor memory (TMEM), operands staged by TMA.
//
// Replaces the reference's Triton matmul_kernel / linear_kernel
// (src/devproc/backend/triton/templates/matmul.py:24-224) for bf16 operands.
//
// C[b] = epilogue(A[b] · B[b]ᵀ); A [M, K] row-major, B [N, K] row-major (both
// K-major, the nn.Linear layout), fp32 accumulation.
//
// Persistent kernel, one CTA per SM, 384 threads in four roles:
//   warp 0  TMA producer: 128×64 A tile + 256×64 B tile per stage (128-byte
//           swizzle), kStages stages guarded by full/empty mbarriers;
//   warp 1  MMA issuer (one thread): 4 × tcgen05.mma (M=128, N=256, K=16) per
//           stage into one of two TMEM accumulators, tcgen05.commit frees the
//           stage and, after the last K block, hands the accumulator over;
//   warp 2  allocates / frees the 512 TMEM columns (2 × 256 fp32 accumulators);
//   warps 4-11 epilogue: two warps per TMEM lane quadrant, each taking half of
//           the columns (each thread owns one accumulator row): bias →
//           activation → residual → cast, staged 64 bytes wide for TMA
//           stores, then release the accumulator so the next tile's MMAs
//           overlap this one.  The common mixes (bias, GELU-tanh, residual
//           add or gate multiply, bf16 or fp32 C) run compile-time
//           specialised loops with the bias columns staged in shared memory;
//           the rest run one general loop.  Every instruction of the epilogue
//           counts: a tile's epilogue is as long as an 8-stage mainloop.
// Tiles are visited in GROUP_M-row bands for L2 reuse of B.  With a stream-K
// workspace the tiles past the last full wave are split by K stage (Sched).
//
// Every mbarrier wait is bounded (%globaltimer); on a timeout the kernel
// records DP_DEVERR_TIMEOUT, all roles stop, the CTA lets in-flight copies and
// MMAs drain for a bounded time, frees its TMEM and returns.
#include <cuda.h>
#include <cstring>

#include "dp_gemm_epilogue.cuh"

namespace dpk_tcgemm {

#ifndef DP_TC_PAIR
#define DP_TC_PAIR 1  // build switch: 0 keeps every GEMM on single-CTA tiles
#endif
constexpr int kMaxDevices = 64;

constexpr int BM = 128, BN = 256, BK = 64;  // per-CTA tile rows, tile columns, K block
constexpr int kEpiWarps = 8;   // two warps per TMEM lane quadrant, each taking half of the columns
constexpr int kThreads = 128 + 32 * kEpiWarps;
constexpr int kGroupM = 8;
constexpr uint32_t kTileABytes = BM * BK * 2;  // 16 KB
constexpr int kTmemCols = 512;                 // two 256-column fp32 accumulators
constexpr uint32_t kEpiBufBytes = 32 * 64;      // one 32-row x 64-byte output chunk (64-byte swizzle)

// Per CTA-group layout.  CG = 1: one CTA computes a 128 x 256 tile and loads
// all 256 rows of B.  CG = 2: a CTA pair computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2; each CTA loads its own 128 rows of A and half of
// B (128 rows), so a stage is 32 KB instead of 48 KB and more stages fit.
template <int CG>
struct Cfg;
// Build switches for tuning: 64-wide K boxes per pipeline stage.  The operand
// ring is 192 KB either way (single CTA: 48 KB per box, pair: 32 KB per box),
// so more boxes per stage means fewer, longer stages and fewer barrier
// round trips per FLOP.
#ifndef DP_TC_PAIR_KBOXES
#define DP_TC_PAIR_KBOXES 2
#endif
#ifndef DP_TC_SINGLE_KBOXES
#define DP_TC_SINGLE_KBOXES 1
#endif
template <>
struct Cfg<1> {
  static constexpr int kKBoxes = DP_TC_SINGLE_KBOXES;  // 64-wide K boxes per stage
  static constexpr int kStages = 4 / DP_TC_SINGLE_KBOXES;
  static constexpr int kEpiBufs = 1;  // output staging chunks per epilogue warp
  static constexpr int kBRows = BN;
};
#ifndef DP_TC_PAIR_STAGES
#define DP_TC_PAIR_STAGES (6 / DP_TC_PAIR_KBOXES)
#endif
#ifndef DP_TC_PAIR_EPI_BUFS
#define DP_TC_PAIR_EPI_BUFS 1
#endif
template <>
struct Cfg<2> {
  static constexpr int kKBoxes = DP_TC_PAIR_KBOXES;
  static constexpr int kStages = DP_TC_PAIR_STAGES;
  static constexpr int kEpiBufs = DP_TC_PAIR_EPI_BUFS;
  static constexpr int kBRows = BN / 2;
};
template <int CG>
constexpr uint32_t b_box_bytes() { return (uint32_t)Cfg<CG>::kBRows * BK * 2; }
template <int CG>
constexpr uint32_t stage_bytes() { return Cfg<CG>::kKBoxes * (kTileABytes + b_box_bytes<CG>()); }
constexpr uint32_t kBiasSliceBytes = 128 * 4;  // one epilogue warp's 128 bias columns as fp32
template <int CG>
constexpr size_t smem_bytes() {  // + 1 KB slack to align the operand stages to 1024 B
  return (size_t)Cfg<CG>::kStages * stage_bytes<CG>() +
         (size_t)kEpiWarps * (Cfg<CG>::kEpiBufs * kEpiBufBytes + kBiasSliceBytes) + 1024;
}

struct Shape {
  int M, N, K, batch;
  int tiles_m, tiles_n, tiles_per_batch, num_tiles, k_blocks;
  int batch2;        // inner batch count (1 = single-level batch)
  int b_mn;          // B is [K, N] (N contiguous) instead of [N, K]
  int tma_store;     // output written by TMA tensor stores from swizzled chunks
  int res_vec;       // residual / gate rows are 16-byte aligned vectors (bf16, f16 or fp32)
  int c_bytes;       // element size of C
  int bcast;         // operands shared by every batch (zero batch strides): 1 A, 2 B
  int tf32;          // operands are fp32 multiplied as TF32 (kind::tf32); else bf16 (kind::f16)
  int box_k;         // K elements per 128-byte operand box: 64 bf16 or 32 fp32
  int last_boxes;    // boxes of the last K stage that lie inside K (the rest are zero fill)
  // Stream-K (sk_ipp > 0): tiles [0, sk_tile0) run whole, sk_tile0 / pairs per
  // pair; the K stages of tiles [sk_tile0, num_tiles) are dealt out as
  // contiguous runs of sk_ipp stages (sk_ipp <= k_blocks) to the sk_pairs pairs.
  int sk_tile0, sk_ipp, sk_pairs;
  // Specialised epilogue (0 = the general one): 1 + bias + 2 * GELU-tanh +
  // 4 * (1 residual add, 2 gate multiply), for bf16 or fp32 C (GELU only with
  // bf16) through TMA, no alpha, residual of C's dtype in 16-byte rows.
  int epi_fast;
};

// One piece of work for a CTA group: K stages [kb0, kb1) of tile t.
// kind 0: the whole tile; 1: a leading or middle run whose raw fp32 partial
// goes to the group's workspace slot; 2: the run that ends the tile, which
// adds the earlier runs' partials before the epilogue.
struct Unit {
  int t, kb0, kb1, kind;
};

// The units of CTA group cid, in processing order: its partial-writing run
// first (the groups that finish those tiles wait for it), then its whole
// tiles, then its remaining runs (whole, or tile-ending).  A group's stream-K
// range covers at most two tiles, and only its last run can stop inside a
// tile, so there is at most one writer and at most two other runs.
struct Sched {
  int nw, ndp, nrest;
  Unit w, r0, r1;
  __device__ __forceinline__ int count() const { return nw + ndp + nrest; }
};

__device__ __forceinline__ Sched make_sched(const Shape &s, int cid, int groups) {
  Sched sc;
  sc.nw = 0;
  sc.nrest = 0;
  sc.w = sc.r0 = sc.r1 = Unit{0, 0, 0, 0};
  if (s.sk_ipp == 0) {
    sc.ndp = cid < s.num_tiles ? (s.num_tiles - 1 - cid) / groups + 1 : 0;
    return sc;
  }
  sc.ndp = s.sk_tile0 / groups;
  const int kb = s.k_blocks;
  const int total = (s.num_tiles - s.sk_tile0) * kb;
  const int i1 = min(cid * s.sk_ipp + s.sk_ipp, total);
  for (int i = cid * s.sk_ipp; i < i1;) {
    const int u = i / kb, k0 = i - u * kb, k1 = min(kb, k0 + (i1 - i));
    const Unit x{s.sk_tile0 + u, k0, k1, k1 < kb ? 1 : (k0 > 0 ? 2 : 0)};
    if (x.kind == 1) {
      sc.w = x;
      sc.nw = 1;
    } else if (sc.nrest == 0) {
      sc.r0 = x;
      sc.nrest = 1;
    } else {
      sc.r1 = x;
      sc.nrest = 2;
    }
    i += k1 - k0;
  }
  return sc;
}

__device__ __forceinline__ Unit sched_unit(const Sched &sc, const Shape &s, int cid, int groups, int j) {
  if (j < sc.nw) return sc.w;
  j -= sc.nw;
  if (j < sc.ndp) return Unit{cid + j * groups, 0, s.k_blocks, 0};
  return j == sc.ndp ? sc.r0 : sc.r1;
}

// ------------------------------------------------------------------ PTX
// Operand maps are 4-D: (cols, rows, inner batch, outer batch); ``z`` is the
// flat batch index, split here by the inner batch count ``b2``.
__device__ __forceinline__ void tma_load_4d(void *smem, const CUtensorMap *map, int x, int y, int z, int b2,
                                            uint64_t *bar) {
  const int zo = z / b2, zi = z - zo * b2;
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(smem_u32(smem)),
      "l"(map), "r"(x), "r"(y), "r"(zi), "r"(zo), "r"(smem_u32(bar))
      : "memory");
}

// Pair form: the completion goes to ``bar`` given as a shared::cluster
// address, here the leader CTA's barrier (both CTAs' bytes are counted there).
__device__ __forceinline__ void tma_load_4d_pair(void *smem, const CUtensorMap *map, int x, int y, int z, int b2,
                                                 uint32_t bar_cluster) {
  const int zo = z / b2, zi = z - zo * b2;
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4, %5}], [%6];" ::"r"(smem_u32(smem)),
      "l"(map), "r"(x), "r"(y), "r"(zi), "r"(zo), "r"(bar_cluster)
      : "memory");
}

// shared::cluster address of the object at ``p`` in CTA ``rank`` of this cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, const void *smem, int x, int y, int z, int b2) {
  const int zo = z / b2, zi = z - zo * b2;
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(map),
               "r"(x), "r"(y), "r"(zi), "r"(zo), "r"(smem_u32(smem))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Byte offset of 16-byte chunk j (0..3) of row r in a 64-byte-swizzled box
// (rows of 64 B; address bits 4-5 XOR bits 7-8).  A warp writing one chunk
// per row touches all 32 banks once per 8 rows.
__device__ __forceinline__ uint32_t swz(int r, int j) { return (uint32_t)(r * 64 + ((j ^ ((r >> 1) & 3)) << 4)); }

__device__ __forceinline__ void prefetch_map(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes, 8-row groups 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                    // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;          // SBO
  d |= (uint64_t)1 << 46;                    // version
  d |= (uint64_t)2 << 61;                    // SWIZZLE_128B
  return d;
}

// Shared-memory descriptor of an MN-major operand (N contiguous), 128-byte
// swizzle: each K row holds 64 N elements (128 B), 8-row groups 1024 B apart
// (SBO), 64-element N chunks 8 KB apart (LBO, one TMA box each).
__device__ __forceinline__ uint64_t smem_desc_mn(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)(8192 >> 4) << 16;          // LBO: next 64-element N chunk
  d |= (uint64_t)(1024 >> 4) << 32;          // SBO: next 8 K rows
  d |= (uint64_t)1 << 46;                    // version
  d |= (uint64_t)2 << 61;                    // SWIZZLE_128B
  return d;
}

// Instruction descriptor: fp32 accumulate, A K-major, B K-major (b_mn = 0)
// or MN-major (b_mn = 1); operand format 1 = BF16 (kind::f16) or 2 = TF32
// (kind::tf32) in both the A and B fields.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n, int b_mn = 0, uint32_t fmt = 1) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

template <int CG>
__device__ __forceinline__ void mma_issue(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate, bool tf32) {
  if constexpr (CG == 1) {
    if (tf32)
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "setp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
          "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
          : "memory");
    else
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "setp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
          "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
          : "memory");
  } else {
    if (tf32)
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "setp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
          "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
          : "memory");
    else
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "setp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
          "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
          : "memory");
  }
}

// Arrive on ``bar`` once the MMAs issued so far have completed; for a pair,
// on the barrier at the same offset in both CTAs.
template <int CG>
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  if constexpr (CG == 1) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
  } else {
    const uint16_t both = 3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(both)
        : "memory");
  }
}

// One lane of a converged warp (the lowest), as elect.sync picks it.  The
// producer and MMA roles run their loops on the whole warp and issue each
// TMA / tcgen05 instruction from the elected lane, so every value the
// instructions take is warp-uniform.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t.reg .b32 R;\n\t"
      "elect.sync R|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void act16(float (&x)[16], int act, bool fast_tanh);

// Out-of-line pieces of the epilogue: element-wise fallbacks and the long
// activations stay out of the unrolled loops, which keeps the kernel's code
// (and so its instruction-fetch stalls) small.
__device__ __noinline__ float load_f32_any(const void *q, int64_t i, int dt) { return load_as_f32(q, i, dt); }
__device__ __noinline__ float gelu_erf_one(float v) { return dp::act_gelu_erf(v); }
__device__ __noinline__ float gelu_tanh_one(float v) { return dp::act_gelu_tanh(v); }
__device__ __noinline__ float silu_one(float v) { return v / (1.0f + expf(-v)); }
// The whole epilogue (alpha, bias, activation, residual, cast) for 16 columns
// n0.. of row m, element by element with bounds checks: rows whose stride or
// base rules out the vector store.
__device__ __noinline__ void store16_generic(const dp_gemm_params &p, void *C, const void *bias, const void *res,
                                             int64_t batch, int64_t m, int64_t n0, const float *x) {
  const dp::Epilogue ep(p, C, bias, res, batch);
  for (int i = 0; i < 16; i += 4) ep.store4(m, n0 + i, x[i], x[i + 1], x[i + 2], x[i + 3]);
}

// Epilogue math on 16 consecutive columns n..n+15 of one row (columns past N
// get bias 0; they are never stored).  One activation switch per call keeps
// the code small enough for the instruction cache.
__device__ __forceinline__ void epi16(float (&x)[16], int64_t n, int N, int epi, const void *bias, int bias_dt,
                                      bool fast_tanh) {
  if (epi & DP_EPI_BIAS) {
    if (bias_dt == DP_BF16 && n + 16 <= N && (reinterpret_cast<uintptr_t>(bias) & 15) == 0 && (n & 7) == 0) {
      const uint4 *bp = reinterpret_cast<const uint4 *>(static_cast<const __nv_bfloat16 *>(bias) + n);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 raw = __ldg(bp + h);
        const __nv_bfloat162 *b2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(b2[e]);
          x[8 * h + 2 * e] += f.x;
          x[8 * h + 2 * e + 1] += f.y;
        }
      }
    } else if (bias_dt == DP_F32 && n + 16 <= N && (reinterpret_cast<uintptr_t>(bias) & 15) == 0 && (n & 3) == 0) {
      const float4 *bp = reinterpret_cast<const float4 *>(static_cast<const float *>(bias) + n);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float4 f = __ldg(bp + h);
        x[4 * h] += f.x;
        x[4 * h + 1] += f.y;
        x[4 * h + 2] += f.z;
        x[4 * h + 3] += f.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (n + e < N) x[e] += load_f32_any(bias, n + e, bias_dt);
    }
  }
  act16(x, epi & (DP_EPI_RELU | DP_EPI_GELU_ERF | DP_EPI_GELU_TANH | DP_EPI_SILU), fast_tanh);
}

// The activation of the epilogue on 16 values (act: at most one DP_EPI_* activation flag).
__device__ __forceinline__ void act16(float (&x)[16], int act, bool fast_tanh) {
  if (act == DP_EPI_RELU) {
#pragma unroll
    for (int e = 0; e < 16; ++e) x[e] = x[e] > 0.0f ? x[e] : (isnan(x[e]) ? x[e] : 0.0f);
  } else if (act == DP_EPI_GELU_ERF) {
#pragma unroll
    for (int e = 0; e < 16; ++e) x[e] = gelu_erf_one(x[e]);
  } else if (act == DP_EPI_GELU_TANH) {
    if (fast_tanh) {
      // 16-bit output: the hardware tanh approximation (relative error far
      // below the output's bf16/fp16 resolution).
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float u = 0.7978845608028654f * (x[e] + 0.044715f * x[e] * x[e] * x[e]);
        float t;
        asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
        x[e] = 0.5f * x[e] * (1.0f + t);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) x[e] = gelu_tanh_one(x[e]);
    }
  } else if (act == DP_EPI_SILU) {
#pragma unroll
    for (int e = 0; e < 16; ++e) x[e] = silu_one(x[e]);
  }
}

// Argmax key of value v in column col: order-preserving bits of v in the high
// word (NaN above everything, -0 as +0) and 0xFFFFFFFF - col in the low word,
// so the largest key belongs to the first column of the maximum (torch.argmax).
__device__ __forceinline__ unsigned long long argmax_key(float v, int64_t col) {
  uint32_t k;
  if (v != v) {
    k = 0xFFFFFFFFu;
  } else {
    const uint32_t u = v == 0.0f ? 0u : __float_as_uint(v);
    k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  return ((unsigned long long)k << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)col);
}

__device__ __forceinline__ float round_to(float v, int dt) {
  if (dt == DP_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dt == DP_F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ void tile_coords(const Shape &s, int t, int &b, int &tm, int &tn) {
  b = t / s.tiles_per_batch;
  const int r = t - b * s.tiles_per_batch;
  const int band = kGroupM * s.tiles_n;
  const int g = r / band;
  const int first_m = g * kGroupM;
  const int gsize = min(kGroupM, s.tiles_m - first_m);
  const int in_band = r - g * band;
  tm = first_m + in_band % gsize;
  tn = in_band / gsize;
}

__device__ __forceinline__ bool aborted(volatile int *flag) { return *flag != 0; }

// A CTA pair's last column tile with at most 128 valid columns (N = 1,152 =
// 4.5 tiles of 256) runs N = 128 MMAs: each CTA then supplies 64 columns of
// B instead of 128, and the MMAs do no work on the missing half.
template <int CG>
__device__ __forceinline__ bool half_width(const Shape &s, int tn) {
  return CG == 2 && !s.b_mn && s.N - tn * BN <= BN / 2;
}

// Waits in 0.2 s slices, re-reading the CTA's abort flag between slices, for
// at most 2 s in total; on giving up records DP_DEVERR_TIMEOUT and raises the
// abort flag so that the other roles stop too.
// kClusterScope: the barrier also collects arrivals from the peer CTA.
// Non-blocking probe of a barrier phase (no suspension of the thread).
template <bool kClusterScope>
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (kClusterScope)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  return ok != 0;
}

template <bool kClusterScope>
__device__ __noinline__ bool wait_or_abort_slow(uint64_t *bar, uint32_t parity, int site, volatile int *flag) {
  for (int slice = 0; slice < 10; ++slice) {
    if (aborted(flag)) return false;
    if (mbar_wait_for<kClusterScope>(bar, parity, 200000000ull)) return true;
  }
  dp_report(DP_DEVERR_TIMEOUT, site);
  *flag = 1;
  return false;
}

template <bool kClusterScope = false>
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, int site, volatile int *flag) {
  // Fast path inline: a phase that is already complete needs no abort-flag
  // read; the bounded slow path is one out-of-line copy.
  if (mbar_test<kClusterScope>(bar, parity)) return true;
  return wait_or_abort_slow<kClusterScope>(bar, parity, site, flag);
}

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int *p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits (at most 2 s, polling every ~0.1 us) until the stream-K arrival
// counter reaches ``target``; on giving up records DP_DEVERR_TIMEOUT and
// raises the abort flag.  Every lane polls, so every lane's later loads are
// ordered after the writers' release.
__device__ __forceinline__ bool counter_wait(const unsigned int *c, unsigned int target, int site,
                                             volatile int *flag) {
  if (ld_acquire_gpu(c) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (aborted(flag)) return false;
    __nanosleep(100);
    if (ld_acquire_gpu(c) >= target) return true;
    if (globaltimer_ns() - t0 > 2000000000ull) break;
  }
  dp_report(DP_DEVERR_TIMEOUT, site);
  *flag = 1;
  return false;
}

// Stream-K partial tiles: per CTA 8 regions (one per epilogue warp) of 32
// column quads x 32 rows of float4, so a warp's stores and loads are
// contiguous 512-byte runs and its region is one 16 KB block.
constexpr int kWarpQuads = 32 * 32;             // float4 per epilogue warp region
constexpr int kCtaQuads = kEpiWarps * kWarpQuads;  // float4 per CTA slot (128 KB)

// Adds NQ column quads (from region quad ql0) of the previous run's
// cumulative partial to x; ``prev`` is the region in global memory or its
// copy in shared memory.
template <int NQ>
__device__ __forceinline__ void add_prev(float (&x)[4 * NQ], const float4 *prev, bool in_smem, int ql0, int lane) {
#pragma unroll
  for (int h = 0; h < NQ; ++h) {
    const float4 *q = prev + (ql0 + h) * 32 + lane;
    const float4 v = in_smem ? *q : __ldcg(q);
    x[4 * h] += v.x;
    x[4 * h + 1] += v.y;
    x[4 * h + 2] += v.z;
    x[4 * h + 3] += v.w;
  }
}

// A warp's 128 bias columns from n0 as fp32 into shared memory (zeros past N).
__device__ __forceinline__ void load_bias_slice(float *bias_s, const void *bias, int dt, int64_t n0, int N, int lane) {
  const int64_t n = n0 + 4 * lane;
  float4 v;
  if (dt == DP_BF16 && n + 4 <= N && (reinterpret_cast<uintptr_t>(bias) & 7) == 0) {
    const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(static_cast<const __nv_bfloat16 *>(bias) + n));
    const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw.x));
    const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw.y));
    v = make_float4(lo.x, lo.y, hi.x, hi.y);
  } else if (dt == DP_F32 && n + 4 <= N && (reinterpret_cast<uintptr_t>(bias) & 15) == 0) {
    v = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(bias) + n));
  } else {
    float t[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) t[i] = n + i < N ? load_f32_any(bias, n + i, dt) : 0.0f;
    v = make_float4(t[0], t[1], t[2], t[3]);
  }
  reinterpret_cast<float4 *>(bias_s)[lane] = v;
  __syncwarp();
}

// Two floats rounded to a bf16 pair (lo in the low half).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t u;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(u) : "f"(hi), "f"(lo));
  return u;
}

// Per-warp arguments of the specialised epilogue for one tile.
struct FastEpi {
  uint32_t tbase;        // TMEM address of this warp's lane quadrant in the accumulator
  int col_lo, c_end;     // first column of the warp's half; end chunk (exclusive)
  int half, lane, q, row0, b, batch2;
  uint8_t *ebuf;         // the warp's 64-byte-wide output staging chunk
  const float *bias_s;   // the warp's bias columns (fp32) in shared memory
  const uint8_t *res;    // the residual / gate row of this thread (nullptr past M)
  const float4 *prev;    // stream-K: the previous run's partial (or nullptr)
  bool prev_smem;
  int nbase;             // first column of the tile
};

// The epilogue of one tile for a fixed mix of steps: CC = 64 / CB columns per
// chunk (one tcgen05.ld, one 64-byte-wide TMA store); a chunk's residual /
// gate words are requested before its staging wait and TMEM load.
template <int CB, bool BIAS, bool GELU, int RES>
__device__ __forceinline__ void epi_fast(const FastEpi f, const CUtensorMap *map_c) {
  constexpr int CC = 64 / CB;
  uint4 rq[4];
  const int c0 = f.col_lo / CC;
#pragma unroll 1
  for (int c = c0; c < f.c_end; ++c) {
    if constexpr (RES != 0) {  // issued first: the staging wait and the TMEM load run under its latency
      if (f.res) {
        const uint4 *src = reinterpret_cast<const uint4 *>(f.res + (size_t)(f.nbase + c * CC) * CB);
#pragma unroll
        for (int h = 0; h < 4; ++h) rq[h] = __ldg(src + h);
      }
    }
    if (f.lane == 0) bulk_wait_read0();  // the previous store has read the staging chunk
    __syncwarp();
    float x[CC];
    {
      uint32_t r[CC];
      if constexpr (CC == 32)
        tmem_ld32(f.tbase + c * CC, r);
      else
        tmem_ld16(f.tbase + c * CC, r);
#pragma unroll
      for (int i = 0; i < CC; ++i) x[i] = __uint_as_float(r[i]);
    }
    if (f.prev) {
      if constexpr (CC == 32)
        add_prev<8>(x, f.prev, f.prev_smem, c * 8 - f.half * 32, f.lane);
      else
        add_prev<4>(x, f.prev, f.prev_smem, c * 4 - f.half * 32, f.lane);
    }
    if constexpr (BIAS) {
      const float4 *bq = reinterpret_cast<const float4 *>(f.bias_s + (c * CC - f.col_lo));
#pragma unroll
      for (int h = 0; h < CC / 4; ++h) {
        const float4 bv = bq[h];
        x[4 * h] += bv.x;
        x[4 * h + 1] += bv.y;
        x[4 * h + 2] += bv.z;
        x[4 * h + 3] += bv.w;
      }
    }
    if constexpr (GELU) {
#pragma unroll
      for (int i = 0; i < CC; ++i) {
        const float u = 0.7978845608028654f * (x[i] + 0.044715f * x[i] * x[i] * x[i]);
        float t;
        asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
        x[i] = 0.5f * x[i] * (1.0f + t);
      }
    }
    if constexpr (RES != 0) {
      if (f.res) {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t w = k == 0 ? rq[h].x : k == 1 ? rq[h].y : k == 2 ? rq[h].z : rq[h].w;
            if constexpr (CB == 2) {  // bf16 pair: low half is the first column
              const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xffff0000u);
              const int i = 8 * h + 2 * k;
              x[i] = RES == 2 ? x[i] * lo : x[i] + lo;
              x[i + 1] = RES == 2 ? x[i + 1] * hi : x[i + 1] + hi;
            } else {
              const float v = __uint_as_float(w);
              const int i = 4 * h + k;
              x[i] = RES == 2 ? x[i] * v : x[i] + v;
            }
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      uint4 packed;
      if constexpr (CB == 2) {
        packed = make_uint4(pack_bf16x2(x[8 * h], x[8 * h + 1]), pack_bf16x2(x[8 * h + 2], x[8 * h + 3]),
                            pack_bf16x2(x[8 * h + 4], x[8 * h + 5]), pack_bf16x2(x[8 * h + 6], x[8 * h + 7]));
      } else {
        packed = make_uint4(__float_as_uint(x[4 * h]), __float_as_uint(x[4 * h + 1]), __float_as_uint(x[4 * h + 2]),
                            __float_as_uint(x[4 * h + 3]));
      }
      *reinterpret_cast<uint4 *>(f.ebuf + swz(f.lane, h)) = packed;
    }
    fence_async_smem();
    __syncwarp();
    if (f.lane == 0) {
      tma_store_4d(map_c, f.ebuf, f.nbase + c * CC, f.row0 + f.q * 32, f.b, f.batch2);
      bulk_commit();
    }
  }
}

// The residual / gate form of epi_fast: the same chunks, finished in
// 16-column pieces (one tcgen05.ld each) to keep the registers of the
// accumulator and the residual words small; the chunk's residual words are
// requested before its staging wait.  Bias, GELU and add-or-multiply are
// warp-uniform run-time choices (one copy of this code, not eight).
// CB 2: bf16 C and residual; 4: fp32.
template <int CB>
__device__ __forceinline__ void epi_fast_res(const FastEpi f, const CUtensorMap *map_c, bool BIAS, bool GELU,
                                             bool MUL) {
  constexpr int CC = 64 / CB;
  constexpr int PW = 16 * CB / 16;  // 16-byte residual words per 16-column piece
  const int c0 = f.col_lo / CC;
#pragma unroll 1
  for (int c = c0; c < f.c_end; ++c) {
    uint4 rq[4];
    if (f.res) {
      const uint4 *src = reinterpret_cast<const uint4 *>(f.res + (size_t)(f.nbase + c * CC) * CB);
#pragma unroll
      for (int h = 0; h < 4; ++h) rq[h] = __ldg(src + h);
    }
    if (f.lane == 0) bulk_wait_read0();  // the previous store has read the staging chunk
    __syncwarp();
#pragma unroll
    for (int piece = 0; piece < CC / 16; ++piece) {
      float x[16];
      {
        uint32_t r[16];
        tmem_ld16(f.tbase + c * CC + piece * 16, r);
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = __uint_as_float(r[i]);
      }
      if (f.prev) add_prev<4>(x, f.prev, f.prev_smem, (c * CC + piece * 16) / 4 - f.half * 32, f.lane);
      if (BIAS) {
        const float4 *bq = reinterpret_cast<const float4 *>(f.bias_s + (c * CC + piece * 16 - f.col_lo));
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float4 bv = bq[h];
          x[4 * h] += bv.x;
          x[4 * h + 1] += bv.y;
          x[4 * h + 2] += bv.z;
          x[4 * h + 3] += bv.w;
        }
      }
      if (GELU) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float u = 0.7978845608028654f * (x[i] + 0.044715f * x[i] * x[i] * x[i]);
          float t;
          asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
          x[i] = 0.5f * x[i] * (1.0f + t);
        }
      }
      if (f.res) {
#pragma unroll
        for (int h = 0; h < PW; ++h) {
          const uint4 w4 = rq[piece * PW + h];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t w = k == 0 ? w4.x : k == 1 ? w4.y : k == 2 ? w4.z : w4.w;
            if constexpr (CB == 2) {  // bf16 pair: low half is the first column
              const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xffff0000u);
              const int i = 8 * h + 2 * k;
              x[i] = MUL ? x[i] * lo : x[i] + lo;
              x[i + 1] = MUL ? x[i + 1] * hi : x[i + 1] + hi;
            } else {
              const float v = __uint_as_float(w);
              const int i = 4 * h + k;
              x[i] = MUL ? x[i] * v : x[i] + v;
            }
          }
        }
      }
      if constexpr (CB == 2) {
#pragma unroll
        for (int h = 0; h < 2; ++h)
          *reinterpret_cast<uint4 *>(f.ebuf + swz(f.lane, piece * 2 + h)) =
              make_uint4(pack_bf16x2(x[8 * h], x[8 * h + 1]), pack_bf16x2(x[8 * h + 2], x[8 * h + 3]),
                         pack_bf16x2(x[8 * h + 4], x[8 * h + 5]), pack_bf16x2(x[8 * h + 6], x[8 * h + 7]));
      } else {
#pragma unroll
        for (int h = 0; h < 4; ++h)
          *reinterpret_cast<uint4 *>(f.ebuf + swz(f.lane, h)) =
              make_uint4(__float_as_uint(x[4 * h]), __float_as_uint(x[4 * h + 1]), __float_as_uint(x[4 * h + 2]),
                         __float_as_uint(x[4 * h + 3]));
      }
    }
    fence_async_smem();
    __syncwarp();
    if (f.lane == 0) {
      tma_store_4d(map_c, f.ebuf, f.nbase + c * CC, f.row0 + f.q * 32, f.b, f.batch2);
      bulk_commit();
    }
  }
}

// CB: bytes per element of C (4: fp32, 2: bf16 / f16); CG: CTAs per tile (1 or 2).
template <int CB, int CG>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_c,
                   const __grid_constant__ dp_gemm_params p, const __grid_constant__ Shape s, void *C,
                   const void *bias, const void *res, float4 *sk_ws,
                   unsigned int *sk_cnt) {
  extern __shared__ uint8_t smem_raw[];
  constexpr int kStages = Cfg<CG>::kStages;
  constexpr int kEpiBufs = Cfg<CG>::kEpiBufs;
  constexpr uint32_t kStageBytes = stage_bytes<CG>();
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2], res_bar[kEpiWarps],
      sm_bar[4];
  __shared__ float2 sm_part[2][4][2][32];  // softmax (max, sum) per accumulator, quadrant, column half, row
  __shared__ uint32_t tmem_base_slot;
  __shared__ int abort_flag;

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  dp::pdl_trigger();
  // The pair's leader (rank 0) issues the MMAs for both CTAs and owns the
  // barriers that gather both CTAs' operand bytes and epilogue releases.
  const uint32_t rank = CG == 2 ? cluster_rank() : 0;
  const int cid = blockIdx.x / CG, nclusters = gridDim.x / CG;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], CG * kEpiWarps);  // one arrival per epilogue warp of each CTA
    }
    for (int i = 0; i < kEpiWarps; ++i) mbar_init(&res_bar[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&sm_bar[i], 64);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_map(&map_a);
    prefetch_map(&map_b);
  }
  if (warp == 2) {
    if constexpr (CG == 1) {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&tmem_base_slot)),
                   "r"(kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    } else {  // warp 2 of both CTAs allocates the pair's columns together
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&tmem_base_slot)),
                   "r"(kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_slot;
  volatile int *flag = &abort_flag;
  dp::pdl_wait();  // set-up above touches no global memory; the previous kernel's results are visible from here

  if (warp == 0) {
    {
      // ---------------- TMA producer (whole warp; the elected lane issues)
      int it = 0;
      const Sched sc = make_sched(s, cid, nclusters);
      for (int j = 0; j < sc.count() && !aborted(flag); ++j) {
        const Unit u = sched_unit(sc, s, cid, nclusters, j);
        int b, tm, tn;
        tile_coords(s, u.t, b, tm, tn);
        const int row0 = tm * BM * CG + (int)rank * BM;               // this CTA's A rows
        // this CTA's B rows (N): half of the pair's columns, 64 instead of 128 on a half-width tile
        const int col0 = tn * BN + (int)rank * (half_width<CG>(s, tn) ? Cfg<CG>::kBRows / 2 : Cfg<CG>::kBRows);
        const int ba = (s.bcast & 1) ? 0 : b, bb = (s.bcast & 2) ? 0 : b;
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++it) {
          const int st = it % kStages;
          if (!wait_or_abort(&empty[st], ((it / kStages) & 1) ^ 1, 300 + st, flag)) break;
          // Stage layout: kKBoxes A boxes (128 rows x 64 K), then kKBoxes B boxes
          // (kBRows x 64 K; MN-major: kBRows / 64 chunks of 64 N x 64 K each).
          uint8_t *sa = smem + st * kStageBytes;
          uint8_t *sb = sa + Cfg<CG>::kKBoxes * kTileABytes;
          uint64_t *bar_local = &full[st];
          uint32_t bar_pair = 0;
          if constexpr (CG == 2) bar_pair = cluster_addr(bar_local, 0);
          auto load = [&](void *dst, const CUtensorMap *map, int x, int y, int z) {
            if constexpr (CG == 1)
              tma_load_4d(dst, map, x, y, z, s.batch2, bar_local);
            else
              tma_load_4d_pair(dst, map, x, y, z, s.batch2, bar_pair);
          };
          if (elect_one()) {
            if constexpr (CG == 1) {
              mbar_arrive_expect_tx(bar_local, kStageBytes);
            } else {
              // Both CTAs' bytes complete on the leader's barrier, which expects them all.
              if (rank == 0) mbar_arrive_expect_tx(bar_local, 2 * kStageBytes);
            }
#pragma unroll
            for (int kh = 0; kh < Cfg<CG>::kKBoxes; ++kh) {
              const int k0 = (kb * Cfg<CG>::kKBoxes + kh) * s.box_k;
              load(sa + kh * kTileABytes, &map_a, k0, row0, ba);
              uint8_t *sbk = sb + kh * b_box_bytes<CG>();
              if (s.b_mn) {
#pragma unroll
                for (int j = 0; j < Cfg<CG>::kBRows / 64; ++j) load(sbk + j * 8192, &map_b, col0 + j * 64, k0, bb);
              } else {
                load(sbk, &map_b, k0, col0, bb);
              }
            }
          }
          __syncwarp();
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------- MMA issuer (the leader CTA's, for a pair; whole warp, the elected lane issues)
      const uint32_t idesc_full = instr_desc(BM * CG, BN, s.b_mn, s.tf32 ? 2u : 1u);
      const uint32_t idesc_half = instr_desc(BM * CG, BN / 2, s.b_mn, s.tf32 ? 2u : 1u);
      const bool tf32 = s.tf32 != 0;
      const bool b_mn = s.b_mn != 0;
      const uint32_t b_kstep = b_mn ? 2048u : 32u;  // bytes per 16-deep K step of B (MN-major: 16 rows of 128 B)
      int it = 0, local = 0;
      const Sched sc = make_sched(s, cid, nclusters);
      for (int j = 0; j < sc.count() && !aborted(flag); ++j, ++local) {
        const Unit u = sched_unit(sc, s, cid, nclusters, j);
        const int a = local & 1;
        int tb, tm, tn;
        tile_coords(s, u.t, tb, tm, tn);
        const uint32_t idesc = half_width<CG>(s, tn) ? idesc_half : idesc_full;
        if (!wait_or_abort<CG == 2>(&acc_empty[a], ((local >> 1) & 1) ^ 1, 310 + a, flag)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + (uint32_t)(a * BN);
        bool ok = true;
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++it) {
          const int st = it % kStages;
          if (!wait_or_abort<CG == 2>(&full[st], (it / kStages) & 1, 320 + st, flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Descriptors of the stage's first K step; later steps add their byte
          // offset >> 4 to the 14-bit address field (shared addresses stay
          // below 256 KB, so the field never carries).
          const uint32_t sa = smem_u32(smem + st * kStageBytes);
          const uint32_t sb = sa + Cfg<CG>::kKBoxes * kTileABytes;
          const uint64_t a_desc0 = smem_desc(sa);
          const uint64_t b_desc0 = b_mn ? smem_desc_mn(sb) : smem_desc(sb);
          const int kh_end = kb + 1 == s.k_blocks ? s.last_boxes : Cfg<CG>::kKBoxes;  // boxes past K hold zeros only
          if (elect_one()) {
#pragma unroll
            for (int kh = 0; kh < Cfg<CG>::kKBoxes; ++kh) {
              if (kh >= kh_end) break;
#pragma unroll
              for (int k = 0; k < BK / 16; ++k) {
                const uint64_t adesc = a_desc0 + (uint64_t)((kh * kTileABytes + k * 32) >> 4);
                const uint64_t bdesc = b_desc0 + (uint64_t)((kh * b_box_bytes<CG>() + k * b_kstep) >> 4);
                mma_issue<CG>(tmem_d, adesc, bdesc, idesc, ((kb - u.kb0) | kh | k) != 0, tf32);
              }
            }
            mma_commit<CG>(&empty[st]);  // stage is free (in both CTAs) once these MMAs have read it
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) mma_commit<CG>(&acc_full[a]);  // accumulator complete
      }
    }
  } else if (warp >= 4) {
    // ---------------- epilogue: warp 4+e owns TMEM lane quadrant q = warp % 4
    // (accumulator rows 32q..32q+31) and column half h = e / 4 of the tile.
    const int e = warp - 4;
    const int q = warp & 3;
    const int half = e >> 2;
    const int row = q * 32 + lane;
    uint8_t *ebuf = smem + kStages * kStageBytes + e * kEpiBufs * kEpiBufBytes;
    float *bias_s = reinterpret_cast<float *>(smem + kStages * kStageBytes + kEpiWarps * kEpiBufs * kEpiBufBytes +
                                              e * kBiasSliceBytes);
    const int rbytes = p.r_dtype == DP_F32 ? 4 : 2;  // residual element size on the vector path
    constexpr int chunk_cols = 64 / CB;  // 16 fp32 or 32 bf16/f16 columns
    uint32_t res_phase = 0;
    int local = 0;
    const uint32_t acc_empty_leader[2] = {CG == 2 ? cluster_addr(&acc_empty[0], 0) : 0u,
                                          CG == 2 ? cluster_addr(&acc_empty[1], 0) : 0u};
    const Sched sc = make_sched(s, cid, nclusters);
    for (int j = 0; j < sc.count(); ++j, ++local) {
      const Unit u = sched_unit(sc, s, cid, nclusters, j);
      const int t = u.t;
      const int a = local & 1;
      // tcgen05.ld is warp-collective: the whole warp continues or stops together.
      const bool got = wait_or_abort(&acc_full[a], (local >> 1) & 1, 330 + a, flag);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      int b, tm, tn;
      tile_coords(s, t, b, tm, tn);
      const int row0 = tm * BM * CG + (int)rank * BM;  // first accumulator row of this CTA
      const int64_t m = (int64_t)row0 + row;
      dp::Epilogue ep(p, C, bias, res, b);
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN);
      const int col_lo = half * (BN / 2);
      const int col_hi = col_lo + BN / 2;
      // Stream-K: a run after the tile's first adds the cumulative partial of
      // the run before it (group cid - 1, which wrote it as its first unit,
      // after its own wait); the counter counts the tile's finished runs.
      const float4 *prev = nullptr;
      bool prev_smem = false;
      if (u.kind == 2 || (u.kind == 1 && u.kb0 > 0)) {
        const int first = (int)(((int64_t)(t - s.sk_tile0) * s.k_blocks) / s.sk_ipp);
        const bool ok = counter_wait(&sk_cnt[t - s.sk_tile0], (unsigned)((cid - first) * CG * kEpiWarps), 360, flag);
        if (!__all_sync(0xffffffffu, ok)) break;
        const float4 *src = sk_ws + ((size_t)(cid - 1) * CG + rank) * kCtaQuads + (size_t)e * kWarpQuads;
        prev = src;
        if (j + 1 == sc.count()) {
          // The group's last unit: its MMAs have finished with the operand
          // ring, so one bulk copy stages this warp's 16 KB region there.
          float4 *dst = reinterpret_cast<float4 *>(smem + (size_t)e * kWarpQuads * 16);
          if (lane == 0) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            mbar_arrive_expect_tx(&res_bar[e], kWarpQuads * 16);
            bulk_g2s(dst, src, kWarpQuads * 16, &res_bar[e]);
          }
          const bool got_prev = wait_or_abort(&res_bar[e], res_phase, 370 + e, flag);
          res_phase ^= 1u;
          if (!__all_sync(0xffffffffu, got_prev)) break;
          prev = dst;
          prev_smem = true;
        }
      }
      if (u.kind == 1) {
        // A run that does not end the tile: the raw fp32 sum so far goes to
        // this group's slot.
        float4 *dst = sk_ws + ((size_t)cid * CG + rank) * kCtaQuads + (size_t)e * kWarpQuads;
#pragma unroll 1
        for (int c = col_lo / 16; c < col_hi / 16; ++c) {
          uint32_t r[16];
          tmem_ld16(tbase + c * 16, r);
          float x[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) x[i] = __uint_as_float(r[i]);
          const int ql0 = c * 4 - half * 32;
          if (prev) add_prev<4>(x, prev, prev_smem, ql0, lane);
#pragma unroll
          for (int h = 0; h < 4; ++h)
            __stcg(dst + (ql0 + h) * 32 + lane, make_float4(x[4 * h], x[4 * h + 1], x[4 * h + 2], x[4 * h + 3]));
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(&sk_cnt[t - s.sk_tile0], 1u);
      } else {
        // Row softmax epilogue: this thread's row is all N (≤ BN) columns of
        // the accumulator, split between the quadrant's two warps.  Each half
        // keeps an online (max, sum) over its columns in log2 units; the pair
        // swaps them through shared memory, guarded by a per-quadrant mbarrier.
        float sm_max = 0.0f, sm_inv = 1.0f, sm_l2 = 0.0f;
        const bool softmax = (p.epilogue & DP_EPI_SOFTMAX) != 0;
        const bool res_mul = (p.epilogue & DP_EPI_MUL) != 0;
        if (softmax) {
          sm_l2 = (p.alpha != 0.0f ? p.alpha : 1.0f) * 1.4426950408889634f;
          float mx = -INFINITY, sum = 0.0f;
#pragma unroll 1
          for (int c = col_lo / 16; c < col_hi / 16; ++c) {
            uint32_t r[16];
            tmem_ld16(tbase + c * 16, r);
            float v[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
              v[e] = ((int64_t)tn * BN + c * 16 + e < s.N) ? __uint_as_float(r[e]) * sm_l2 : -INFINITY;
            float t[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) t[e] = fmaxf(v[e], v[e + 8]);
#pragma unroll
            for (int e = 0; e < 4; ++e) t[e] = fmaxf(t[e], t[e + 4]);
            const float nm = fmaxf(mx, fmaxf(fmaxf(t[0], t[2]), fmaxf(t[1], t[3])));
            if (nm == -INFINITY) continue;
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              s0 += ex2_approx(v[e] - nm);
              s1 += ex2_approx(v[e + 1] - nm);
            }
            sum = sum * ex2_approx(mx - nm) + (s0 + s1);
            mx = nm;
          }
          sm_part[a][q][half][lane] = make_float2(mx, sum);
          mbar_arrive(&sm_bar[q]);
          const bool ok = wait_or_abort(&sm_bar[q], local & 1, 350 + q, flag);
          if (!__all_sync(0xffffffffu, ok)) break;
          const float2 o = sm_part[a][q][half ^ 1][lane];
          const float gm = fmaxf(mx, o.x);
          const float tot = (mx == -INFINITY ? 0.0f : sum * ex2_approx(mx - gm)) +
                            (o.x == -INFINITY ? 0.0f : o.y * ex2_approx(o.x - gm));
          sm_max = gm;
          sm_inv = 1.0f / tot;
        }
        if (p.epilogue & DP_EPI_ARGMAX) {
          // The row's largest key over this warp's columns, then one atomicMax per row.
          unsigned long long best = 0ull;
          const int epi = p.epilogue & ~DP_EPI_ARGMAX;
#pragma unroll 1
          for (int c = col_lo / 16; c < col_hi / 16; ++c) {
            const int64_t nb = (int64_t)tn * BN + c * 16;
            if (nb >= s.N) break;
            uint32_t r[16];
            tmem_ld16(tbase + c * 16, r);
            float x[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] = __uint_as_float(r[e]) * (p.alpha != 0.0f ? p.alpha : 1.0f);
            if (epi) epi16(x, nb, s.N, epi, bias, p.bias_dtype, p.c_dtype != DP_F32);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              if (nb + e >= s.N) break;
              float v = x[e];
              if ((epi & (DP_EPI_RESIDUAL | DP_EPI_MUL)) && m < s.M) {
                const float rv = load_f32_any(res, ep.r_off + m * p.ldr + nb + e, p.r_dtype);
                v = res_mul ? v * rv : v + rv;
              }
              const unsigned long long k = argmax_key(round_to(v, p.c_dtype), nb + e);
              best = k > best ? k : best;
            }
          }
          if (m < s.M && best) atomicMax(static_cast<unsigned long long *>(C) + ep.c_off + m, best);
        } else if (s.epi_fast) {
          constexpr int CC = 64 / CB;
          const int k = s.epi_fast - 1;  // bias + 2 * GELU + 4 * residual mode
          FastEpi f;
          f.tbase = tbase;
          f.col_lo = col_lo;
          const int ncols = (int)min((int64_t)BN, (int64_t)s.N - (int64_t)tn * BN);
          f.c_end = min(col_hi, (ncols + CC - 1) / CC * CC) / CC;
          f.half = half;
          f.lane = lane;
          f.q = q;
          f.row0 = row0;
          f.b = b;
          f.batch2 = s.batch2;
          f.ebuf = ebuf;
          f.bias_s = bias_s;
          f.res = (k >= 4 && m < s.M)
                      ? static_cast<const uint8_t *>(res) + (size_t)(ep.r_off + m * p.ldr) * CB
                      : nullptr;
          f.prev = prev;
          f.prev_smem = prev_smem;
          f.nbase = tn * BN;
          if (k & 1) load_bias_slice(bias_s, bias, p.bias_dtype, (int64_t)tn * BN + col_lo, s.N, lane);
          switch (k) {
            case 0: epi_fast<CB, false, false, 0>(f, &map_c); break;
            case 1: epi_fast<CB, true, false, 0>(f, &map_c); break;
            case 2: epi_fast<CB, false, true, 0>(f, &map_c); break;
            case 3: epi_fast<CB, true, true, 0>(f, &map_c); break;
            default: epi_fast_res<CB>(f, &map_c, k & 1, (k >> 1) & 1, k >= 8); break;
          }
        } else if (s.tma_store) {
          bool stop = false;
          // 16 columns per step, 64-byte-wide output chunks (SPC steps each)
          // staged in shared memory and written by TMA.  The warp's bias
          // columns are read once per tile into shared memory; the residual /
          // gate values of the next step are loaded while this step runs.
          constexpr int SPC = chunk_cols / 16;
          const int ncols = (int)min((int64_t)BN, (int64_t)s.N - (int64_t)tn * BN);
          const int g_begin = col_lo / 16;
          const int g_end = min(col_hi, (ncols + chunk_cols - 1) / chunk_cols * chunk_cols) / 16;
          const int act = p.epilogue & (DP_EPI_RELU | DP_EPI_GELU_ERF | DP_EPI_GELU_TANH | DP_EPI_SILU);
          const bool has_bias = (p.epilogue & DP_EPI_BIAS) != 0 && !softmax;
          const bool has_res = (p.epilogue & (DP_EPI_RESIDUAL | DP_EPI_MUL)) != 0;
          const bool res_rows = has_res && s.res_vec && m < s.M;
          if (has_bias) load_bias_slice(bias_s, bias, p.bias_dtype, (int64_t)tn * BN + col_lo, s.N, lane);
          // Raw residual words of step g (16 values: 32 bytes of bf16 / f16 or 64 of fp32).
          auto res_load = [&](int g, uint4(&w)[4]) {
            const int64_t nb = (int64_t)tn * BN + g * 16;
            if (res_rows && nb + 16 <= s.N) {
              const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(res) +
                                                                 (ep.r_off + m * p.ldr + nb) * rbytes);
              w[0] = __ldg(src);
              w[1] = __ldg(src + 1);
              if (rbytes == 4) {
                w[2] = __ldg(src + 2);
                w[3] = __ldg(src + 3);
              }
            }
          };
          uint4 rqa[4], rqb[4];
          if (g_begin < g_end) res_load(g_begin, rqa);
          uint8_t *buf = ebuf;
#pragma unroll 1
          for (int g = g_begin; g < g_end; ++g) {
            const int step = (g - g_begin) % SPC;
            const int64_t nb = (int64_t)tn * BN + g * 16;
            if (step == 0) {
              buf = ebuf + ((g - g_begin) / SPC % kEpiBufs) * kEpiBufBytes;
              if (lane == 0) {  // the store that last read ``buf`` is done with it
                if constexpr (kEpiBufs == 2) bulk_wait_read1();
                else bulk_wait_read0();
              }
              __syncwarp();
            }
            if (g + 1 < g_end) res_load(g + 1, rqb);
            uint32_t r[16];
            tmem_ld16(tbase + g * 16, r);
            float x[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) x[i] = __uint_as_float(r[i]);
            if (prev) add_prev<4>(x, prev, prev_smem, g * 4 - half * 32, lane);
            if (softmax) {
#pragma unroll
              for (int i = 0; i < 16; ++i) x[i] = ex2_approx(fmaf(x[i], sm_l2, -sm_max)) * sm_inv;
            } else {
              if (p.alpha != 0.0f) {
#pragma unroll
                for (int i = 0; i < 16; ++i) x[i] *= p.alpha;
              }
              if (has_bias) {
                const float4 *bq = reinterpret_cast<const float4 *>(bias_s + (g * 16 - col_lo));
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                  const float4 bv = bq[h];
                  x[4 * h] += bv.x;
                  x[4 * h + 1] += bv.y;
                  x[4 * h + 2] += bv.z;
                  x[4 * h + 3] += bv.w;
                }
              }
              if (act) act16(x, act, CB == 2);
            }
            if (has_res && m < s.M) {
              float rv[16];
              if (s.res_vec && nb + 16 <= s.N) {
                if (rbytes == 4) {
#pragma unroll
                  for (int h = 0; h < 4; ++h) {
                    rv[4 * h] = __uint_as_float(rqa[h].x);
                    rv[4 * h + 1] = __uint_as_float(rqa[h].y);
                    rv[4 * h + 2] = __uint_as_float(rqa[h].z);
                    rv[4 * h + 3] = __uint_as_float(rqa[h].w);
                  }
                } else {
#pragma unroll
                  for (int h = 0; h < 2; ++h) {
                    const uint32_t wd[4] = {rqa[h].x, rqa[h].y, rqa[h].z, rqa[h].w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                      float2 f;
                      if (p.r_dtype == DP_BF16)
                        f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&wd[k]));
                      else
                        f = __half22float2(*reinterpret_cast<const __half2 *>(&wd[k]));
                      rv[8 * h + 2 * k] = f.x;
                      rv[8 * h + 2 * k + 1] = f.y;
                    }
                  }
                }
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                  rv[i] = nb + i < s.N ? load_f32_any(res, ep.r_off + m * p.ldr + nb + i, p.r_dtype) : 0.0f;
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) x[i] = res_mul ? x[i] * rv[i] : x[i] + rv[i];
            }
#pragma unroll
            for (int h = 0; h < 4; ++h) rqa[h] = rqb[h];
            // This step's 16 columns are 16-byte units step*2.. (16-bit C) or step*4.. (fp32 C) of the chunk.
            if constexpr (CB == 4) {
#pragma unroll
              for (int h = 0; h < 4; ++h)
                *reinterpret_cast<float4 *>(buf + swz(lane, step * 4 + h)) =
                    make_float4(x[4 * h], x[4 * h + 1], x[4 * h + 2], x[4 * h + 3]);
            } else {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                uint4 packed;
                uint32_t *pw = reinterpret_cast<uint32_t *>(&packed);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  if (p.c_dtype == DP_BF16) {
                    const __nv_bfloat162 v2 = __floats2bfloat162_rn(x[8 * h + 2 * k], x[8 * h + 2 * k + 1]);
                    pw[k] = *reinterpret_cast<const uint32_t *>(&v2);
                  } else {
                    const __half2 v2 = __floats2half2_rn(x[8 * h + 2 * k], x[8 * h + 2 * k + 1]);
                    pw[k] = *reinterpret_cast<const uint32_t *>(&v2);
                  }
                }
                *reinterpret_cast<uint4 *>(buf + swz(lane, step * 2 + h)) = packed;
              }
            }
            if (step == SPC - 1) {
              fence_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_4d(&map_c, buf, (int)(nb - (SPC - 1) * 16), row0 + q * 32, b, s.batch2);
                bulk_commit();
              }
            }
          }
          if (stop) break;
        } else {
#pragma unroll 1
          for (int c = col_lo / 16; c < col_hi / 16; ++c) {
            uint32_t r[16];
            tmem_ld16(tbase + c * 16, r);
            float x[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] = __uint_as_float(r[e]);
            if (prev) add_prev<4>(x, prev, prev_smem, c * 4 - half * 32, lane);
            const int64_t n0 = (int64_t)tn * BN + c * 16;
            if (m < s.M && n0 < s.N) store16_generic(p, C, bias, res, b, m, n0, x);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {  // this warp has read its part of accumulator a
        if constexpr (CG == 1)
          mbar_arrive(&acc_empty[a]);
        else
          mbar_arrive_cluster(acc_empty_leader[a]);
      }
    }
    if (lane == 0) bulk_wait_all();  // every TMA store of this warp has landed
  }

  __syncthreads();
  if (aborted(flag) && threadIdx.x == 0) {
    // Let in-flight TMA copies and MMAs finish (bounded) before TMEM and
    // shared memory go away.
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // neither CTA leaves while the pair's MMAs may touch it
  if (warp == 2) {
    tc_fence_after();
    if constexpr (CG == 1)
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                   : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                   : "memory");
  }
}

// ------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// rows × cols matrix of ``dt`` (row stride ld elements) in a two-level batch:
// outer count ``b1`` with stride ``s1``, inner count ``b2`` with stride ``s2``
// (elements); boxes of box_cols × box_rows with 128-byte swizzle.
int make_map(CUtensorMap *map, const void *base, int dt, int64_t rows, int64_t cols, int64_t ld, int64_t b1,
             int64_t s1, int64_t b2, int64_t s2, int box_cols, int box_rows,
             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  DP_REQUIRE(fn != nullptr, DP_ERR_CUDA, "gemm: cuTensorMapEncodeTiled unavailable");
  const int eb = dp::dtype_bytes(dt);
  CUtensorMapDataType t = dt == DP_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                          : dt == DP_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  // Unused batch levels get a harmless stride (one matrix further on).
  const int64_t mat = rows * ld;
  if (b2 <= 1) s2 = mat;
  if (b1 <= 1) s1 = (b2 > 1 ? b2 * s2 : mat);
  cuuint64_t dims[4] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)(b2 > 1 ? b2 : 1),
                        (cuuint64_t)(b1 > 1 ? b1 : 1)};
  cuuint64_t strides[3] = {(cuuint64_t)(ld * eb), (cuuint64_t)(s2 * eb), (cuuint64_t)(s1 * eb)};
  cuuint32_t box[4] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, t, 4, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  DP_REQUIRE(r == CUDA_SUCCESS, DP_ERR_CUDA, "gemm: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return DP_OK;
}

// Build switches for the stream-K cost model (units: one K stage of a tile).
#ifndef DP_SK_FIX_STAGES
#define DP_SK_FIX_STAGES 2.0
#endif
#ifndef DP_SK_PART_STAGES
#define DP_SK_PART_STAGES 1.5
#endif

// Stream-K plan for a launch of ``groups`` CTA groups: the tiles past the last
// full wave are split by K stage when each group's share is at least half a
// tile (so a tile has at most three runs) and the modelled time - waves x
// stages, plus the share, a fixed cost and a cost per partial handed on - is
// at most 0.9 of the whole-tile schedule's.
struct SkPlan {
  int tile0 = 0, ipp = 0;
  int64_t counter_bytes = 0, bytes = 0;
};
SkPlan streamk_plan(const Shape &s, int groups, int cg, int epilogue) {
  SkPlan k;
  if (epilogue & (DP_EPI_SOFTMAX | DP_EPI_ARGMAX)) return k;
  const int kb = s.k_blocks, rem = s.num_tiles % groups, waves = s.num_tiles / groups;
  if (rem == 0 || kb < 4) return k;
  const int ipp = (rem * kb + groups - 1) / groups;  // <= kb, since rem < groups
  if (2 * ipp < kb) return k;                           // at most three runs per tile (a chain of two partials)
  const int runs = (kb + ipp - 1) / ipp + 1;            // runs per split tile, at most
  const double t_tiles = (double)(waves + 1) * kb;
  const double t_sk = (double)waves * kb + ipp + DP_SK_FIX_STAGES + DP_SK_PART_STAGES * (runs - 1);
  if (t_sk > 0.9 * t_tiles) return k;
  k.tile0 = waves * groups;
  k.ipp = ipp;
  k.counter_bytes = ((int64_t)rem * 4 + 255) / 256 * 256;
  k.bytes = k.counter_bytes + (int64_t)groups * cg * 64 * 128 * 16;
  return k;
}

}  // namespace dpk_tcgemm

namespace dp {

int64_t gemm_streamk_workspace_bound(const dp_gemm_params &p) {
  using namespace dpk_tcgemm;
  const int64_t tiles = (p.M + BM - 1) / BM * ((p.N + BN - 1) / BN) * (p.batch > 0 ? p.batch : 1);
  return (tiles * 4 + 255) / 256 * 256 + (int64_t)num_sms() * 64 * 128 * 16;
}

// Switches ``s`` to the stream-K schedule when the plan picks it and the
// caller's workspace holds it: counters first (cleared here), then one
// partial-tile slot per CTA group.
int use_streamk(dpk_tcgemm::Shape &s, int groups, int cg, int epilogue, void *workspace, int64_t bytes,
                cudaStream_t stream, float4 *&ws, unsigned int *&cnt) {
  if (!workspace) return DP_OK;
  DP_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, DP_ERR_ARG,
             "gemm: the stream-K workspace must be 16-byte aligned");
  const dpk_tcgemm::SkPlan k = dpk_tcgemm::streamk_plan(s, groups, cg, epilogue);
  if (!k.ipp || bytes < k.bytes) return DP_OK;
  s.sk_tile0 = k.tile0;
  s.sk_ipp = k.ipp;
  s.sk_pairs = groups;
  cnt = static_cast<unsigned int *>(workspace);
  ws = reinterpret_cast<float4 *>(static_cast<uint8_t *>(workspace) + k.counter_bytes);
  DP_CHECK_CUDA(cudaMemsetAsync(workspace, 0, (size_t)k.counter_bytes, stream));
  return DP_OK;
}

int launch_gemm_tc(const dp_gemm_params &p, const void *A, const void *B, void *C, const void *bias,
                   const void *res, cudaStream_t stream, void *sk_workspace, int64_t sk_bytes) {
  using namespace dpk_tcgemm;
  CUtensorMap ma, mb, mc;
  memset(&mc, 0, sizeof(mc));
  const int64_t b2 = p.batch2 > 1 ? p.batch2 : 1;
  const int64_t b1 = p.batch / b2;
  // An operand with zero batch strides is one matrix shared by every batch:
  // its map has no batch extent and the kernel reads it at batch 0.
  auto shared = [&](int64_t s1, int64_t s2) { return p.batch > 1 && s1 == 0 && (b2 == 1 || s2 == 0); };
  const bool a_sh = shared(p.stride_a, p.stride_a2), b_sh = shared(p.stride_b, p.stride_b2);
  const bool tf32 = p.a_dtype == DP_TF32;
  const int ab_dt = tf32 ? DP_F32 : DP_BF16;
  const int box_k = tf32 ? 32 : 64;  // K elements per 128-byte box
  int st = a_sh ? make_map(&ma, A, ab_dt, p.M, p.K, p.lda, 1, 0, 1, 0, box_k, BM)
                : make_map(&ma, A, ab_dt, p.M, p.K, p.lda, b1, p.stride_a, b2, p.stride_a2, box_k, BM);
  if (st != DP_OK) return st;
  const bool b_mn = p.b_layout == DP_B_KN;
  const int64_t mb1 = b_sh ? 1 : b1, mb2 = b_sh ? 1 : b2;
  if (b_mn)  // [K, N], N contiguous: boxes of 64 N × 64 K (the same for a CTA pair)
    st = make_map(&mb, B, DP_BF16, p.K, p.N, p.ldb, mb1, p.stride_b, mb2, p.stride_b2, 64, BK);
  else
    st = make_map(&mb, B, ab_dt, p.N, p.K, p.ldb, mb1, p.stride_b, mb2, p.stride_b2, box_k, BN);
  if (st != DP_OK) return st;
  const int cb = dtype_bytes(p.c_dtype);
  auto al16 = [](const void *q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  const bool argmax = (p.epilogue & DP_EPI_ARGMAX) != 0;  // C holds one uint64 key per row
  const bool tma_store = !argmax && (p.ldc * cb) % 16 == 0 && (p.batch == 1 || (p.stride_c * cb) % 16 == 0) &&
                         (b2 == 1 || (p.stride_c2 * cb) % 16 == 0) && al16(C) && (cb == 4 || cb == 2);
  if (tma_store) {
    st = make_map(&mc, C, p.c_dtype, p.M, p.N, p.ldc, b1, p.stride_c, b2, p.stride_c2, 64 / cb, 32,
                  CU_TENSOR_MAP_SWIZZLE_64B);
    if (st != DP_OK) return st;
  }
  // Residual / gate rows read as 16-byte vectors (any of bf16, f16, fp32; a
  // residual shared by every batch has zero batch strides).
  const int rb = (p.epilogue & (DP_EPI_RESIDUAL | DP_EPI_MUL)) ? dtype_bytes(p.r_dtype) : 0;
  const bool res_vec = (rb == 2 || rb == 4) && (p.ldr * rb) % 16 == 0 && (p.batch == 1 || (p.stride_r * rb) % 16 == 0) &&
                       (b2 == 1 || (p.stride_r2 * rb) % 16 == 0) && al16(res);
  // A CTA pair per 256-row tile when both operands fill more than one CTA's share.
  const int cg = (DP_TC_PAIR && p.M > BM && p.N > BN / 2) ? 2 : 1;
  Shape s;
  s.M = (int)p.M;
  s.N = (int)p.N;
  s.K = (int)p.K;
  s.batch = (int)p.batch;
  s.tiles_m = (int)((p.M + BM * cg - 1) / (BM * cg));
  s.tiles_n = (int)((p.N + BN - 1) / BN);
  s.tiles_per_batch = s.tiles_m * s.tiles_n;
  s.num_tiles = s.tiles_per_batch * s.batch;
  const int kstep = box_k * (cg == 2 ? Cfg<2>::kKBoxes : Cfg<1>::kKBoxes);  // K per stage
  s.k_blocks = (int)((p.K + kstep - 1) / kstep);
  s.last_boxes = (int)((p.K - (int64_t)(s.k_blocks - 1) * kstep + box_k - 1) / box_k);
  DP_REQUIRE(tma_store || !(p.epilogue & DP_EPI_SOFTMAX), DP_ERR_UNSUPPORTED,
             "gemm: the softmax epilogue needs a 16-byte aligned C with 16-byte row strides");
  s.batch2 = (int)b2;
  s.b_mn = b_mn ? 1 : 0;
  s.tma_store = tma_store ? 1 : 0;
  s.res_vec = res_vec ? 1 : 0;
  {
    const int epi = p.epilogue;
    const bool gelu = (epi & DP_EPI_GELU_TANH) != 0;
    const int resm = (epi & DP_EPI_RESIDUAL) ? 1 : (epi & DP_EPI_MUL) ? 2 : 0;
    bool fast = tma_store && p.alpha == 0.0f &&
                !(epi & (DP_EPI_SOFTMAX | DP_EPI_ARGMAX | DP_EPI_RELU | DP_EPI_GELU_ERF | DP_EPI_SILU)) &&
                ((cb == 2 && p.c_dtype == DP_BF16) || (cb == 4 && !gelu));
    if (resm) fast = fast && res_vec && p.r_dtype == p.c_dtype && p.N % (64 / cb) == 0;
    s.epi_fast = fast ? 1 + ((epi & DP_EPI_BIAS) ? 1 : 0) + (gelu ? 2 : 0) + 4 * resm : 0;
  }
  s.c_bytes = cb;
  s.bcast = (a_sh ? 1 : 0) | (b_sh ? 2 : 0);
  s.tf32 = tf32 ? 1 : 0;
  s.box_k = box_k;
  s.sk_tile0 = s.sk_ipp = s.sk_pairs = 0;
  DP_REQUIRE(p.N < (1ll << 31) && p.K < (1ll << 31), DP_ERR_UNSUPPORTED, "gemm: N or K too large");
  if (cg == 2 && !b_mn) {  // each CTA of the pair loads 128 rows of B
    st = make_map(&mb, B, ab_dt, p.N, p.K, p.ldb, mb1, p.stride_b, mb2, p.stride_b2, box_k, Cfg<2>::kBRows);
    if (st != DP_OK) return st;
  }
  int dev = 0;
  DP_CHECK_CUDA(cudaGetDevice(&dev));
  DP_REQUIRE(dev >= 0 && dev < kMaxDevices, DP_ERR_UNSUPPORTED, "gemm: device ordinal out of range");
  if (cg == 1) {
    static bool attr_set[kMaxDevices] = {};
    if (!attr_set[dev]) {
      DP_CHECK_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem_bytes<1>()));
      DP_CHECK_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<2, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem_bytes<1>()));
      attr_set[dev] = true;
    }
    int grid = num_sms();
    float4 *ws = nullptr;
    unsigned int *cnt = nullptr;
    st = use_streamk(s, grid, 1, p.epilogue, sk_workspace, sk_bytes, stream, ws, cnt);
    if (st != DP_OK) return st;
    if (!s.sk_ipp && grid > s.num_tiles) grid = s.num_tiles;
    if (cb == 4)
      dp::launch_k(tc_gemm_kernel<4, 1>, grid, kThreads, smem_bytes<1>(), stream, ma, mb, mc, p, s, C, bias, res, ws, cnt);
    else
      dp::launch_k(tc_gemm_kernel<2, 1>, grid, kThreads, smem_bytes<1>(), stream, ma, mb, mc, p, s, C, bias, res, ws, cnt);
  } else {
    auto kern = cb == 4 ? tc_gemm_kernel<4, 2> : tc_gemm_kernel<2, 2>;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // as dp::launch_k
    attr[1].val.programmaticStreamSerializationAllowed = DP_PDL ? 1 : 0;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes<2>();
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;  // the cluster shape (the occupancy query)
    // Co-resident pairs (clusters never straddle a GPC, so this can be below SMs / 2).
    static int pairs[kMaxDevices][2] = {};
    int &np = pairs[dev][cb == 4 ? 0 : 1];
    if (np == 0) {
      DP_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes<2>()));
      cfg.gridDim = dim3(2 * (num_sms() / 2));
      int n = 0;
      DP_CHECK_CUDA(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
      DP_REQUIRE(n > 0, DP_ERR_CUDA, "gemm: no CTA pair fits on this device");
      np = n;
    }
    float4 *ws = nullptr;
    unsigned int *cnt = nullptr;
    st = use_streamk(s, np, 2, p.epilogue, sk_workspace, sk_bytes, stream, ws, cnt);
    if (st != DP_OK) return st;
    const int grid_pairs = (s.sk_ipp || np < s.num_tiles) ? np : s.num_tiles;
    cfg.gridDim = dim3(2 * grid_pairs);
    cfg.numAttrs = 2;  // cluster shape + programmatic dependent launch
    DP_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, p, s, C, bias, res, ws, cnt));
  }
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

}  // namespace dp
