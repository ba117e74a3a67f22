// Fused attention on the 5th-generation tensor cores:
//   O = softmax(scale · Q·Kᵀ) · V, bf16 operands, fp32 scores and accumulation,
// the scores never leave the SM.
//
// One persistent CTA per SM works through items of 128 query rows of one
// (batch, key/value head); the query heads that share a key/value head are
// stacked rows (grouped-query attention), so every item reads one K / V
// stream.  Per item the key/value blocks of 64 keys stream through two TMA
// rings (K and V, so a K slot frees as soon as its Q·Kᵀ is done), and five
// roles run concurrently:
//   warp 0   TMA producer: the Q tile once per item, then K blocks;
//   warp 3   TMA producer of the V blocks;
//   warp 1   MMA issuer (one thread): S_j = Q·K_jᵀ into one of two TMEM
//            score buffers, issued one block ahead, then O += P_j·V_j into
//            the TMEM output accumulator; Q is released right after the
//            item's last Q·Kᵀ so the next item's Q loads under the tail;
//   warp 2   allocates / frees the 512 TMEM columns;
//   warps 4-7 softmax and epilogue, one query row per thread: read S_j from
//            TMEM, keep the row's running max m and sum l in log2 units,
//            write P_j = 2^(s − m) as bf16 into one of two 128-byte-swizzled
//            shared tiles (so P_{j+1} is written while P_j·V_j runs), and at
//            the end O / l → bf16 → global.
// Head dims ≤ 128 use 128-key blocks in attn_split_kernel (below), whose
// eight softmax warps split every block's keys in two halves.
// The running max is raised lazily (only when a block's max exceeds it by
// more than 2^8): P then stays ≤ 256, exact in bf16's exponent range, and O
// and l are rescaled by 2^(m_old − m_new) only on those rare blocks.
//
// Every mbarrier wait is bounded (%globaltimer); on a timeout the kernel
// records DP_DEVERR_TIMEOUT, all roles stop, in-flight copies and MMAs get a
// bounded time to drain, TMEM is freed and the kernel returns.
#include <cuda.h>
#include <cstring>

#include "dp_common.cuh"

namespace dpk_attn {

constexpr int BM = 128;        // query rows per item
constexpr int kMaxStages = 4;
constexpr int kTmemCols = 512;
constexpr uint32_t kQBox = BM * 128;    // 16 KB: 128 rows × 64 bf16
constexpr uint32_t kPBox = BM * 128;    // 16 KB: 128 rows × 64 bf16 keys of P
// Keys per block: 64 (attn_kernel), or 128 for head dims ≤ 128
// (attn_split_kernel: half the per-block hand-offs; two 128-column score
// buffers and two ≤ 128-column half outputs fit the 512 TMEM columns, and two
// stages still fit shared memory).
template <int BKV>
struct Blk {
  static constexpr int kSCols = BKV;                    // one score buffer: BKV fp32 columns
  static constexpr uint32_t kKVBox = BKV * 128;         // one 64-column box of K or V: BKV rows × 128 B
  static constexpr uint32_t kPBytes = (BKV / 64) * kPBox;  // one P tile: BKV / 64 swizzle atoms along the keys
  // 64-key blocks (head dims above 128) add four output-epilogue warps (8-11),
  // so the softmax warps start the next item while an item's O is written.
  static constexpr bool kSepEpi = BKV == 64;
  static constexpr int kThreads = kSepEpi ? 384 : 256;
};

struct Shape {
  int R;        // query rows per (batch, kv head): group · L
  int L, S, D, Dv;
  int nd, ndv;  // 64-wide boxes of D (Q, K) and of Dv (V)
  int ks;       // K = 16 MMA steps covering D
  int dvp;      // PV MMA N: Dv rounded up to 16
  int stages;
  int o_tma;    // 1: O leaves through shared memory and TMA tensor stores (map_o)
  int tiles_r, items, kv_blocks, heads_kv, group;
  uint32_t stage_bytes, q_bytes;
  float scale_log2;
  int64_t o_sb, o_sh, o_sl;
};

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void tma_load(void *dst, const CUtensorMap *map, int x, int y, int z, int w,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(su32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(su32(bar))
      : "memory");
}

// TMA tensor store of a 64-column × 32-row box from 128-byte-swizzled shared memory
__device__ __forceinline__ void tma_store(const CUtensorMap *map, const void *src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(map),
               "r"(x), "r"(y), "r"(z), "r"(w), "r"(su32(src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint64_t desc_k(uint32_t addr) {  // K-major, 128-byte swizzle, 8-row groups 1024 B
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// MN-major, 64-element N chunks (V boxes) ``chunk`` bytes apart
__device__ __forceinline__ uint64_t desc_mn(uint32_t addr, uint32_t chunk) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(chunk >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__host__ __device__ constexpr uint32_t idesc(int m, int n, int b_mn) {  // bf16 × bf16 → fp32
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// tcgen05.ld without the wait: several loads in flight, one tcgen05.wait::ld after them
__device__ __forceinline__ void tld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// two columns of a warp's 32 TMEM lanes (one value pair per row)
__device__ __forceinline__ void tst2(uint32_t taddr, float a, float b) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(__float_as_uint(a)),
               "r"(__float_as_uint(b))
               : "memory");
}
__device__ __forceinline__ void tld2(uint32_t taddr, float &a, float &b) {
  uint32_t x, y;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(x), "=r"(y) : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  a = __uint_as_float(x);
  b = __uint_as_float(y);
}
__device__ __forceinline__ void tst16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool aborted(volatile int *f) { return *f != 0; }

// One lane of a converged warp, as elect.sync picks it: the producer and MMA
// roles run their loops on the whole warp and issue each TMA / tcgen05
// instruction from the elected lane, so the instructions' operands are
// warp-uniform (a single-lane loop measured slower in the GEMM).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t.reg .b32 R;\n\t"
      "elect.sync R|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ bool mbar_done(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// 0.2 s slices re-reading the abort flag, 2 s in total; on giving up records
// DP_DEVERR_TIMEOUT and raises the abort flag.  A phase already complete
// returns without reading the flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, int site, volatile int *flag) {
  if (mbar_done(bar, parity)) return true;
  for (int slice = 0; slice < 10; ++slice) {
    if (aborted(flag)) return false;
    if (mbar_wait_for(bar, parity, 200000000ull)) return true;
  }
  dp_report(DP_DEVERR_TIMEOUT, site);
  *flag = 1;
  return false;
}

__device__ __forceinline__ void item_coords(const Shape &s, int item, int &b, int &hk, int &rt) {
  rt = item % s.tiles_r;
  const int bh = item / s.tiles_r;
  hk = bh % s.heads_kv;
  b = bh / s.heads_kv;
}

template <int BKV>
__global__ void __launch_bounds__(Blk<BKV>::kThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const Shape s, __nv_bfloat16 *__restrict__ out) {
  constexpr int kSCols = Blk<BKV>::kSCols;
  constexpr uint32_t kKVBox = Blk<BKV>::kKVBox;
  constexpr uint32_t kPBytes = Blk<BKV>::kPBytes;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full, q_empty, k_full[kMaxStages], k_empty[kMaxStages], v_full[kMaxStages],
      v_empty[kMaxStages], s_full[2], s_free[2], p_full[2], p_free[2], o_full, o_free, l_full[2];
  __shared__ float l_rows[2][BM];  // separate epilogue: each row's softmax sum, by item parity
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sq = smem;
  uint8_t *sp = sq + s.q_bytes;
  uint8_t *sk_ring = sp + 2 * kPBytes;  // two P tiles: softmax writes P_{j+1} while P_j is still being read
  uint8_t *sv_ring = sk_ring + (size_t)s.stages * s.nd * kKVBox;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  dp::pdl_trigger();

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    for (int i = 0; i < kMaxStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 4);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(&o_full, 1);
    mbar_init(&o_free, 4);
    for (int i = 0; i < 2; ++i) mbar_init(&l_full[i], 4);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&map_q) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&map_k) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&map_v) : "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t t_o = tmem + 2 * kSCols;  // output accumulator columns
  volatile int *flag = &abort_flag;
  dp::pdl_wait();  // set-up above touches no global memory; the previous kernel's results are visible from here
  const int nb = s.kv_blocks;
  // With two ring stages a K / V slot and a score / P buffer share their index
  // (both are the block count mod 2), so the producers wait on the score and
  // P barriers instead of separate K / V "empty" barriers.
  const bool merged = s.stages == 2;
  // Separate output-epilogue warps (64-key blocks) when an item has at least
  // three key blocks: the third block's wait on P buffer (jg - 2) then implies
  // the P·V that waited for the previous item's epilogue, so a row-sum slot
  // (l_rows, by item parity) is never rewritten before it is read.
  const bool sep_epi = Blk<BKV>::kSepEpi && nb >= 3;
  // O / l → bf16 → global for the rows of one item (thread = row); waits for
  // O, releases it.  False when a wait gave up.
  auto attn_epilogue_rows = [&](int b, int hk, int rt, int row, uint32_t lane_off, int lane, float l,
                                int local) -> bool {
    const bool of = wait_or_abort(&o_full, local & 1, 580, flag);
    if (!__all_sync(0xffffffffu, of)) return false;
    fence_after();
    const int r = rt * BM + row;
    const float inv = 1.0f / l;
    __nv_bfloat16 *orow = nullptr;
    if (r < s.R) {
      const int hq = hk * s.group + r / s.L, pos = r % s.L;
      orow = out + (int64_t)b * s.o_sb + (int64_t)hq * s.o_sh + (int64_t)pos * s.o_sl;
    }
    for (int c = 0; c < s.dvp / 16; ++c) {
      uint32_t rr[16];
      tld16(t_o + lane_off + c * 16, rr);
      if (orow) {
        __nv_bfloat162 h[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          h[e] = __floats2bfloat162_rn(__uint_as_float(rr[2 * e]) * inv, __uint_as_float(rr[2 * e + 1]) * inv);
        const int c0 = c * 16;
        if (c0 + 16 <= s.Dv) {
          uint4 *dst = reinterpret_cast<uint4 *>(orow + c0);
          dst[0] = *reinterpret_cast<const uint4 *>(&h[0]);
          dst[1] = *reinterpret_cast<const uint4 *>(&h[4]);
        } else {
          const __nv_bfloat16 *hv = reinterpret_cast<const __nv_bfloat16 *>(h);
          for (int e = 0; c0 + e < s.Dv; ++e) orow[c0 + e] = hv[e];
        }
      }
    }
    fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&o_free);
    return true;
  };

  if (warp == 0) {
    {
      // ---------------- TMA producer (whole warp; the elected lane issues)
      int it = 0, local = 0;
      for (int item = blockIdx.x; item < s.items && !aborted(flag); item += gridDim.x, ++local) {
        int b, hk, rt;
        item_coords(s, item, b, hk, rt);
        if (!wait_or_abort(&q_empty, (local & 1) ^ 1, 500, flag)) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&q_full, s.q_bytes);
          for (int x = 0; x < s.nd; ++x) tma_load(sq + x * kQBox, &map_q, x * 64, rt * BM, hk, b, &q_full);
        }
        __syncwarp();
        bool ok = true;
        for (int j = 0; j < nb; ++j, ++it) {
          const int st = it % s.stages;
          // Two stages: slot st is free once S of block it − 2 (score buffer st) is complete,
          // so the K ring waits on s_full and the MMA thread commits one barrier less per block.
          const bool free_k = merged ? (it < 2 || wait_or_abort(&s_full[st], ((it - 2) >> 1) & 1, 510 + st, flag))
                                     : wait_or_abort(&k_empty[st], ((it / s.stages) & 1) ^ 1, 510 + st, flag);
          if (!free_k) {
            ok = false;
            break;
          }
          uint8_t *sk = sk_ring + (size_t)st * s.nd * kKVBox;
          if (elect_one()) {
            mbar_arrive_expect_tx(&k_full[st], (uint32_t)s.nd * kKVBox);
            for (int x = 0; x < s.nd; ++x) tma_load(sk + x * kKVBox, &map_k, x * 64, j * BKV, hk, b, &k_full[st]);
          }
          __syncwarp();
        }
        if (!ok) break;
      }
    }
  } else if (warp == 3) {
    {
      // ---------------- TMA producer of V: its own ring, so a K slot frees as
      // soon as its Q·Kᵀ is done instead of waiting for the block's P·V
      int it = 0;
      for (int item = blockIdx.x; item < s.items && !aborted(flag); item += gridDim.x) {
        int b, hk, rt;
        item_coords(s, item, b, hk, rt);
        bool ok = true;
        for (int j = 0; j < nb; ++j, ++it) {
          const int st = it % s.stages;
          // Two stages: slot st is free once P·V of block it − 2 (P buffer st) is complete.
          const bool free_v = merged ? (it < 2 || wait_or_abort(&p_free[st], ((it - 2) >> 1) & 1, 515 + st, flag))
                                     : wait_or_abort(&v_empty[st], ((it / s.stages) & 1) ^ 1, 515 + st, flag);
          if (!free_v) {
            ok = false;
            break;
          }
          uint8_t *sv = sv_ring + (size_t)st * s.ndv * kKVBox;
          if (elect_one()) {
            mbar_arrive_expect_tx(&v_full[st], (uint32_t)s.ndv * kKVBox);
            for (int x = 0; x < s.ndv; ++x) tma_load(sv + x * kKVBox, &map_v, x * 64, j * BKV, hk, b, &v_full[st]);
          }
          __syncwarp();
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    {
      // ---------------- MMA issuer (whole warp; the elected lane issues)
      const uint32_t id_s = idesc(BM, BKV, 0), id_pv = idesc(BM, s.dvp, 1);
      int it = 0, jg = 0, local = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < s.items && ok && !aborted(flag); item += gridDim.x, ++local) {
        if (!wait_or_abort(&q_full, local & 1, 520, flag)) break;
        fence_after();
        const uint32_t aq = su32(sq);
        auto issue_s = [&](int j) -> bool {  // S_j into score buffer (jg + j) % 2
          const int itj = it + j, jgj = jg + j, st = itj % s.stages, sb = jgj & 1;
          if (!wait_or_abort(&k_full[st], (itj / s.stages) & 1, 530 + st, flag)) return false;
          if (!wait_or_abort(&s_free[sb], ((jgj >> 1) & 1) ^ 1, 540 + sb, flag)) return false;
          fence_after();
          const uint32_t ak = su32(sk_ring + (size_t)st * s.nd * kKVBox);
          if (elect_one()) {
            for (int k = 0; k < s.ks; ++k) {
              const uint32_t box = (uint32_t)(k >> 2), sub = (uint32_t)(k & 3) * 32;  // 64-wide box, 16-wide step
              mma(tmem + sb * kSCols, desc_k(aq + box * kQBox + sub), desc_k(ak + box * kKVBox + sub), id_s,
                  k > 0 ? 1u : 0u);
            }
            commit(&s_full[sb]);
            if (!merged) commit(&k_empty[st]);  // K_j is read once S_j is complete
            if (j == nb - 1) commit(&q_empty);  // the item's last read of Q: the next Q may load now
          }
          __syncwarp();
          return true;
        };
        if (!issue_s(0)) break;
        for (int j = 0; j < nb; ++j) {
          if (j + 1 < nb && !issue_s(j + 1)) {
            ok = false;
            break;
          }
          const int itj = it + j, jgj = jg + j, st = itj % s.stages, pb = jgj & 1;
          // the previous item's epilogue has read O before this item's first P·V overwrites it
          if (j == 0 && !wait_or_abort(&o_free, (local & 1) ^ 1, 521, flag)) {
            ok = false;
            break;
          }
          if (!wait_or_abort(&p_full[pb], (jgj >> 1) & 1, 550 + pb, flag)) {
            ok = false;
            break;
          }
          if (!wait_or_abort(&v_full[st], (itj / s.stages) & 1, 535 + st, flag)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t ap = su32(sp + pb * kPBytes), av = su32(sv_ring + (size_t)st * s.ndv * kKVBox);
          if (elect_one()) {
            for (int k = 0; k < BKV / 16; ++k)  // 16 keys per step: P atom k / 4, V rows k·16
              mma(t_o, desc_k(ap + (uint32_t)(k >> 2) * kPBox + (uint32_t)(k & 3) * 32),
                  desc_mn(av + k * 2048, kKVBox), id_pv, (j > 0 || k > 0) ? 1u : 0u);
            if (!merged) commit(&v_empty[st]);  // V_j is read
            commit(&p_free[pb]);    // P_j is read and O holds blocks ≤ j
          }
          __syncwarp();
        }
        it += nb;
        jg += nb;
        if (!ok) break;
        if (elect_one()) commit(&o_full);
        __syncwarp();
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------- softmax (+ epilogue unless sep_epi): thread = query row (warp - 4)·32 + lane
    const int q4 = warp - 4;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    int jg = 0, local = 0;
    bool ok = true;
    const bool sc_neg = s.scale_log2 < 0.0f;
    const float sc = fabsf(s.scale_log2);
    for (int item = blockIdx.x; item < s.items && ok; item += gridDim.x, ++local) {
      int b, hk, rt;
      item_coords(s, item, b, hk, rt);
      float m = -INFINITY, l = 0.0f;
      for (int j = 0; j < nb; ++j, ++jg) {
        const int sb = jg & 1;
        const bool got = wait_or_abort(&s_full[sb], (jg >> 1) & 1, 560 + sb, flag);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        fence_after();
        float v[BKV];
        {
          uint32_t r[BKV / 16][16];
#pragma unroll
          for (int c = 0; c < BKV / 16; ++c) tld16_async(tmem + lane_off + sb * kSCols + c * 16, r[c]);
          tld_wait();  // all four loads in flight together
#pragma unroll
          for (int c = 0; c < BKV / 16; ++c)
#pragma unroll
            for (int e = 0; e < 16; ++e) v[c * 16 + e] = __uint_as_float(r[c][e]);
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[sb]);  // this score buffer may take S_{j+2}
        const int k0 = j * BKV;
        float t8[8];
        // The max runs on raw scores and the scale folds into the exponent's FMA;
        // a negative scale negates the scores first (one warp-uniform branch).
        if (sc_neg) {
#pragma unroll
          for (int e = 0; e < BKV; ++e) v[e] = -v[e];
        }
        if (k0 + BKV > s.S) {  // the last, partial key block only
#pragma unroll
          for (int e = 0; e < BKV; ++e) v[e] = (k0 + e < s.S) ? v[e] : -INFINITY;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {  // tree max: short dependency chains
          const float a = fmaxf(fmaxf(v[e], v[e + 8]), fmaxf(v[e + 16], v[e + 24]));
          const float b2 = fmaxf(fmaxf(v[e + 32], v[e + 40]), fmaxf(v[e + 48], v[e + 56]));
          t8[e] = fmaxf(a, b2);
          if constexpr (BKV == 128) {
            const float c = fmaxf(fmaxf(v[e + 64], v[e + 72]), fmaxf(v[e + 80], v[e + 88]));
            const float d = fmaxf(fmaxf(v[e + 96], v[e + 104]), fmaxf(v[e + 112], v[e + 120]));
            t8[e] = fmaxf(t8[e], fmaxf(c, d));
          }
        }
        const float mx = sc * fmaxf(fmaxf(fmaxf(t8[0], t8[1]), fmaxf(t8[2], t8[3])),
                                    fmaxf(fmaxf(t8[4], t8[5]), fmaxf(t8[6], t8[7])));
        // This block's P tile is free once the P·V of block jg − 2 is complete.
        const int pb = jg & 1;
        if (jg >= 2) {
          const bool pf = wait_or_abort(&p_free[pb], ((jg >> 1) & 1) ^ 1, 570 + pb, flag);
          if (!__all_sync(0xffffffffu, pf)) {
            ok = false;
            break;
          }
          fence_after();
        }
        if (j == 0) {
          m = mx;
        } else if (__any_sync(0xffffffffu, mx > m + 8.0f)) {
          // O must hold every issued block (P·V of block jg − 1 complete) before it is
          // rescaled.  tcgen05.ld / st are warp-collective: the whole warp rescales its
          // rows, rows whose max did not grow by more than 2^8 by a factor of 1.
          const int prev = jg - 1;
          const bool pv = wait_or_abort(&p_free[prev & 1], (prev >> 1) & 1, 575, flag);
          if (!__all_sync(0xffffffffu, pv)) {
            ok = false;
            break;
          }
          fence_after();
          float alpha = 1.0f;
          if (mx > m + 8.0f) {
            alpha = ex2(m - mx);
            l *= alpha;
            m = mx;
          }
          for (int c = 0; c < s.dvp / 16; ++c) {
            uint32_t r[16];
            tld16(t_o + lane_off + c * 16, r);
#pragma unroll
            for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tst16(t_o + lane_off + c * 16, r);
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        // P_j row as bf16 into the 128-byte-swizzled K-major tile
        // (BKV / 64 swizzle atoms of 64 keys, each 128 rows × 128 B)
        uint8_t *prow = sp + pb * kPBytes + row * 128;
        const float nm = -m;  // p = 2^(score · scale − m), one FFMA and one ex2
        float part[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int ch = 0; ch < BKV / 8; ++ch) {
          uint32_t w[4];
          float acc = 0.0f;
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float p0 = ex2(fmaf(v[ch * 8 + 2 * h], sc, nm)), p1 = ex2(fmaf(v[ch * 8 + 2 * h + 1], sc, nm));
            acc += p0 + p1;
            __nv_bfloat162 bb = __floats2bfloat162_rn(p0, p1);
            w[h] = *reinterpret_cast<uint32_t *>(&bb);
          }
          part[ch & 7] += acc;  // eight independent partial sums
          *reinterpret_cast<uint4 *>(prow + (ch >> 3) * kPBox + (((ch & 7) ^ (row & 7)) << 4)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
        l += ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[pb]);
      }
      if (!ok) break;
      if (sep_epi) {
        // hand the row sums to the epilogue warps (they read O once o_full completes)
        l_rows[local & 1][row] = l;
        __syncwarp();
        if (lane == 0) mbar_arrive(&l_full[local & 1]);
        continue;
      }
      if (!attn_epilogue_rows(b, hk, rt, row, lane_off, lane, l, local)) {
        ok = false;
        break;
      }
    }
  } else if (Blk<BKV>::kSepEpi && warp >= 8) {
    // ---------------- output epilogue warps: thread = query row (warp - 8)·32 + lane
    const int q4 = warp - 8;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    int local = 0;
    for (int item = blockIdx.x; item < s.items && sep_epi && !aborted(flag); item += gridDim.x, ++local) {
      int b, hk, rt;
      item_coords(s, item, b, hk, rt);
      const bool lf = wait_or_abort(&l_full[local & 1], (local >> 1) & 1, 585 + (local & 1), flag);
      if (!__all_sync(0xffffffffu, lf)) break;
      if (!attn_epilogue_rows(b, hk, rt, row, lane_off, lane, l_rows[local & 1][row], local)) break;
    }
  }

  __syncthreads();
  if (aborted(flag) && threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();  // let copies and MMAs in flight drain (bounded)
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  __syncthreads();
  if (warp == 2) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// 128-key blocks (head dims ≤ 128) with each block's keys split between two
// softmax warps per TMEM lane quadrant: warps 4-7 take keys 0-63 of every
// block, warps 8-11 keys 64-127.  One softmax warp per SM sub-partition was
// latency-bound (about 1,700 cycles of dependent issue plus 1,000 of MUFU per
// 128-key block); two warps per sub-partition can overlap each other's
// latencies (measured: a few per cent at the ViT shape).  Each half
// keeps its own running max m_h, sum l_h and output accumulator O_h in TMEM
// (O_h += P_h · V_h over its 64 keys), so the halves never exchange anything
// per block; at the end of an item they exchange (m_h, l_h) once and every
// warp writes its share of the columns of
//   O = (2^(m_0 − M)·O_0 + 2^(m_1 − M)·O_1) / (2^(m_0 − M)·l_0 + 2^(m_1 − M)·l_1),
// M = max(m_0, m_1).  A half that has seen no valid key yet (short key
// ranges) has m_h = −∞, l_h = 0, O_h = 0 and weight 0.
//   TMEM: two 128-column score buffers (S_j = Q·K_jᵀ, N = 128, both halves at
//   once) and O_0, O_1 at columns 256 and 384.
//   Shared memory: the Q tile, two P tiles of 128 keys and the K / V rings, as
//   in attn_kernel; P tile pb holds P_0 in its first 64-key atom and P_1 in its
//   second.  After an item's last block the
//   tile the next item writes first carries the (m, l) exchange and the other
//   tile stages the output for the per-warp TMA tensor stores.
// ---------------------------------------------------------------------------
constexpr int kSplitThreads = 384;
// Outputs of at most 112 columns (kSep): four more warps (12-15) combine and
// store each item's output, so the softmax warps go on to the next item as
// soon as their last P block is written.  A softmax warp leaves its (m, l) in
// columns 126-127 of its half's O_h in TMEM (the P·V MMAs and rescales touch
// only the first dvp columns); the epilogue warps read both halves' values and
// O_0, O_1, release the accumulators and then store the rows.
constexpr int kSepThreads = 512, kSepMaxDv = 112, kMLCol = 126, kSepChunks = kSepMaxDv / 16;

template <bool kSep>
__global__ void __launch_bounds__(kSep ? kSepThreads : kSplitThreads, 1)
    attn_split_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                      const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                      const Shape s, __nv_bfloat16 *__restrict__ out) {
  constexpr int BKV = 128;
  constexpr uint32_t kKVBox = Blk<BKV>::kKVBox;
  constexpr uint32_t kPBytes = Blk<BKV>::kPBytes;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full, q_empty, k_full[kMaxStages], k_empty[kMaxStages], v_full[kMaxStages],
      v_empty[kMaxStages], s_full[2], s_free[2], p_full[2][2], p_free[2][2], o_full, o_free, xch[4], xdone,
      lrdy;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sq = smem;
  uint8_t *sp = sq + s.q_bytes;
  uint8_t *sk_ring = sp + 2 * kPBytes;
  uint8_t *sv_ring = sk_ring + (size_t)s.stages * s.nd * kKVBox;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  dp::pdl_trigger();

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    for (int i = 0; i < kMaxStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 8);
      for (int h = 0; h < 2; ++h) {
        mbar_init(&p_full[i][h], 4);
        mbar_init(&p_free[i][h], 1);
      }
    }
    mbar_init(&o_full, 1);
    mbar_init(&o_free, kSep ? 4 : 8);  // the epilogue warps, or all eight softmax warps
    mbar_init(&lrdy, 8);
    for (int i = 0; i < 4; ++i) mbar_init(&xch[i], 2);
    mbar_init(&xdone, 8);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&map_q) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&map_k) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&map_v) : "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int *flag = &abort_flag;
  dp::pdl_wait();
  const int nb = s.kv_blocks;
  const bool merged = s.stages == 2;  // K / V slot index = score / P buffer index (block count mod 2)

  if (warp == 0) {
    // ---------------- TMA producer of Q and K (whole warp; the elected lane issues)
    int it = 0, local = 0;
    for (int item = blockIdx.x; item < s.items && !aborted(flag); item += gridDim.x, ++local) {
      int b, hk, rt;
      item_coords(s, item, b, hk, rt);
      if (!wait_or_abort(&q_empty, (local & 1) ^ 1, 600, flag)) break;
      if (elect_one()) {
        mbar_arrive_expect_tx(&q_full, s.q_bytes);
        for (int x = 0; x < s.nd; ++x) tma_load(sq + x * kQBox, &map_q, x * 64, rt * BM, hk, b, &q_full);
      }
      __syncwarp();
      bool ok = true;
      for (int j = 0; j < nb; ++j, ++it) {
        const int st = it % s.stages;
        const bool free_k = merged ? (it < 2 || wait_or_abort(&s_full[st], ((it - 2) >> 1) & 1, 610 + st, flag))
                                   : wait_or_abort(&k_empty[st], ((it / s.stages) & 1) ^ 1, 610 + st, flag);
        if (!free_k) {
          ok = false;
          break;
        }
        uint8_t *sk = sk_ring + (size_t)st * s.nd * kKVBox;
        if (elect_one()) {
          mbar_arrive_expect_tx(&k_full[st], (uint32_t)s.nd * kKVBox);
          for (int x = 0; x < s.nd; ++x) tma_load(sk + x * kKVBox, &map_k, x * 64, j * BKV, hk, b, &k_full[st]);
        }
        __syncwarp();
      }
      if (!ok) break;
    }
  } else if (warp == 3) {
    // ---------------- TMA producer of V
    int it = 0;
    for (int item = blockIdx.x; item < s.items && !aborted(flag); item += gridDim.x) {
      int b, hk, rt;
      item_coords(s, item, b, hk, rt);
      bool ok = true;
      for (int j = 0; j < nb; ++j, ++it) {
        const int st = it % s.stages;
        // two stages: slot st is free once both halves' P·V of block it − 2 are complete
        const uint32_t ph = ((it - 2) >> 1) & 1;
        const bool free_v = merged ? (it < 2 || (wait_or_abort(&p_free[st][0], ph, 615 + st, flag) &&
                                                 wait_or_abort(&p_free[st][1], ph, 615 + st, flag)))
                                   : wait_or_abort(&v_empty[st], ((it / s.stages) & 1) ^ 1, 615 + st, flag);
        if (!free_v) {
          ok = false;
          break;
        }
        uint8_t *sv = sv_ring + (size_t)st * s.ndv * kKVBox;
        if (elect_one()) {
          mbar_arrive_expect_tx(&v_full[st], (uint32_t)s.ndv * kKVBox);
          for (int x = 0; x < s.ndv; ++x) tma_load(sv + x * kKVBox, &map_v, x * 64, j * BKV, hk, b, &v_full[st]);
        }
        __syncwarp();
      }
      if (!ok) break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (whole warp; the elected lane issues)
    const uint32_t id_s = idesc(BM, BKV, 0), id_pv = idesc(BM, s.dvp, 1);
    const uint32_t aq = su32(sq);
    auto issue_s = [&](int itj, int jgj, bool last) -> bool {
      const int st = itj % s.stages, sb = jgj & 1;
      if (!wait_or_abort(&k_full[st], (itj / s.stages) & 1, 630 + st, flag)) return false;
      if (!wait_or_abort(&s_free[sb], ((jgj >> 1) & 1) ^ 1, 640 + sb, flag)) return false;
      fence_after();
      const uint32_t ak = su32(sk_ring + (size_t)st * s.nd * kKVBox);
      if (elect_one()) {
        for (int k = 0; k < s.ks; ++k) {
          const uint32_t box = (uint32_t)(k >> 2), sub = (uint32_t)(k & 3) * 32;
          mma(tmem + sb * BKV, desc_k(aq + box * kQBox + sub), desc_k(ak + box * kKVBox + sub), id_s,
              k > 0 ? 1u : 0u);
        }
        commit(&s_full[sb]);
        if (!merged) commit(&k_empty[st]);
        if (last) commit(&q_empty);
      }
      __syncwarp();
      return true;
    };
    // An item's first S is issued after the previous item's last P·V: issuing
    // it before made that P·V wait for this item's Q load (about 6,000 cycles
    // from issue to arrival at the ViT shape; 8% slower).
    int it = 0, jg = 0, local = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < s.items && ok && !aborted(flag); item += gridDim.x, ++local) {
      if (!wait_or_abort(&q_full, local & 1, 620, flag)) break;
      fence_after();
      if (!issue_s(it, jg, nb == 1)) break;
      for (int j = 0; j < nb && ok; ++j) {
        if (j + 1 < nb && !(ok = issue_s(it + j + 1, jg + j + 1, j + 1 == nb - 1))) break;
        const int itj = it + j, jgj = jg + j, st = itj % s.stages, pb = jgj & 1;
        // every warp has read the previous item's O_0 and O_1
        if (j == 0 && !(ok = wait_or_abort(&o_free, (local & 1) ^ 1, 621, flag))) break;
        if (!(ok = wait_or_abort(&v_full[st], (itj / s.stages) & 1, 635 + st, flag))) break;
        const uint32_t av = su32(sv_ring + (size_t)st * s.ndv * kKVBox);
        for (int h = 0; h < 2 && ok; ++h) {
          if (!(ok = wait_or_abort(&p_full[pb][h], (jgj >> 1) & 1, 650 + 2 * pb + h, flag))) break;
          fence_after();
          const uint32_t ap = su32(sp + pb * kPBytes + h * kPBox);
          if (elect_one()) {
            for (int k = 0; k < 4; ++k)  // 16 keys per step: V rows (4h + k)·16
              mma(tmem + 256 + h * 128, desc_k(ap + (uint32_t)k * 32), desc_mn(av + (4 * h + k) * 2048, kKVBox),
                  id_pv, (j > 0 || k > 0) ? 1u : 0u);
            commit(&p_free[pb][h]);  // P_h of block j is read, O_h holds blocks ≤ j
            if (h == 1 && !merged) commit(&v_empty[st]);
          }
          __syncwarp();
        }
      }
      it += nb;
      jg += nb;
      if (!ok) break;
      if (elect_one()) commit(&o_full);
      __syncwarp();
    }
  } else if (warp >= 4 && warp < 12) {
    // ---------------- softmax halves (and the epilogue without kSep): thread = query row q4·32 + lane
    const int h = (warp - 4) >> 2, q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t t_oh = tmem + 256 + (uint32_t)h * 128 + lane_off;  // this half's output accumulator
    const bool sc_neg = s.scale_log2 < 0.0f;
    const float sc = fabsf(s.scale_log2);
    const int nchunk = s.dvp / 16, c_lo = 4 * h, c_hi = min(4 * h + 4, nchunk);  // this warp's output columns
    int jg = 0, local = 0, staged = -1;  // staged: the P tile this warp's TMA store still reads
    bool ok = true;
    auto wait_staged = [&](int tile) {
      if (staged == tile) {
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        staged = -1;
      }
    };
    for (int item = blockIdx.x; item < s.items && ok; item += gridDim.x, ++local) {
      int b, hk, rt;
      item_coords(s, item, b, hk, rt);
      float m = -INFINITY, l = 0.0f;
      for (int j = 0; j < nb; ++j, ++jg) {
        const int sb = jg & 1;
        if (!__all_sync(0xffffffffu, wait_or_abort(&s_full[sb], (jg >> 1) & 1, 660 + sb, flag))) {
          ok = false;
          break;
        }
        fence_after();
        float v[64];
        {
          uint32_t r[4][16];
#pragma unroll
          for (int c = 0; c < 4; ++c) tld16_async(tmem + lane_off + sb * BKV + h * 64 + c * 16, r[c]);
          tld_wait();
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 16; ++e) v[c * 16 + e] = __uint_as_float(r[c][e]);
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[sb]);
        const int k0 = j * BKV + h * 64;
        if (sc_neg) {
#pragma unroll
          for (int e = 0; e < 64; ++e) v[e] = -v[e];
        }
        if (k0 + 64 > s.S) {  // the partial tail of the key range (possibly all of this half)
#pragma unroll
          for (int e = 0; e < 64; ++e) v[e] = (k0 + e < s.S) ? v[e] : -INFINITY;
        }
        float t8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a = fmaxf(fmaxf(v[e], v[e + 8]), fmaxf(v[e + 16], v[e + 24]));
          const float b2 = fmaxf(fmaxf(v[e + 32], v[e + 40]), fmaxf(v[e + 48], v[e + 56]));
          t8[e] = fmaxf(a, b2);
        }
        const float mx = sc * fmaxf(fmaxf(fmaxf(t8[0], t8[1]), fmaxf(t8[2], t8[3])),
                                    fmaxf(fmaxf(t8[4], t8[5]), fmaxf(t8[6], t8[7])));
        const int pb = jg & 1;
        if (jg >= 2) {  // P_h of block jg − 2 (same tile) has been read
          if (!__all_sync(0xffffffffu, wait_or_abort(&p_free[pb][h], ((jg >> 1) & 1) ^ 1, 670 + pb, flag))) {
            ok = false;
            break;
          }
          fence_after();
        }
        if (j == 0) {
          m = mx;
        } else if (__any_sync(0xffffffffu, mx > m + 8.0f)) {
          // O_h holds every issued block of this half before it is rescaled
          const int prev = jg - 1;
          if (!__all_sync(0xffffffffu, wait_or_abort(&p_free[prev & 1][h], (prev >> 1) & 1, 675, flag))) {
            ok = false;
            break;
          }
          fence_after();
          float alpha = 1.0f;
          if (mx > m + 8.0f) {
            alpha = ex2(m - mx);  // 0 while this half had no valid key (m = −∞)
            l *= alpha;
            m = mx;
          }
          for (int c = 0; c < nchunk; ++c) {
            uint32_t r[16];
            tld16(t_oh + c * 16, r);
#pragma unroll
            for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tst16(t_oh + c * 16, r);
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        if (!kSep && j == 0 && local > 0) {
          // the previous item's (m, l) exchange in this tile has been read by every warp
          if (!__all_sync(0xffffffffu, wait_or_abort(&xdone, (local - 1) & 1, 680, flag))) {
            ok = false;
            break;
          }
        }
        wait_staged(pb);
        uint8_t *prow = sp + pb * kPBytes + h * kPBox + row * 128;
        const float nm = m == -INFINITY ? 0.0f : -m;  // p = 2^(score · scale − m); 0 for masked keys
        float part[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          uint32_t w[4];
          float acc = 0.0f;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float p0 = ex2(fmaf(v[ch * 8 + 2 * q], sc, nm)), p1 = ex2(fmaf(v[ch * 8 + 2 * q + 1], sc, nm));
            acc += p0 + p1;
            __nv_bfloat162 bb = __floats2bfloat162_rn(p0, p1);
            w[q] = *reinterpret_cast<uint32_t *>(&bb);
          }
          part[ch] = acc;
          *reinterpret_cast<uint4 *>(prow + ((ch ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        l += ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[pb][h]);
      }
      if (!ok) break;
      if constexpr (kSep) {
        // (m, l) to the epilogue warps, once they have read the previous item's
        if (local > 0 && !__all_sync(0xffffffffu, wait_or_abort(&o_free, (local - 1) & 1, 694, flag))) {
          ok = false;
          break;
        }
        fence_after();
        tst2(tmem + lane_off + 256 + (uint32_t)h * 128 + kMLCol, m, l);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&lrdy);
        continue;
      }

      // ---- end of the item: exchange (m, l) through the tile the next item writes first
      const int xt = jg & 1, yt = xt ^ 1;  // exchange tile, staging tile
      if (jg >= 2) {  // this half's P in the exchange tile (block jg − 2) has been read
        if (!__all_sync(0xffffffffu, wait_or_abort(&p_free[xt][h], ((jg - 2) >> 1) & 1, 685, flag))) {
          ok = false;
          break;
        }
        fence_after();
      }
      wait_staged(xt);
      *reinterpret_cast<float2 *>(sp + xt * kPBytes + h * kPBox + row * 128) = make_float2(m, l);
      __syncwarp();
      if (lane == 0) mbar_arrive(&xch[q4]);
      if (!__all_sync(0xffffffffu, wait_or_abort(&xch[q4], local & 1, 686 + q4, flag))) {
        ok = false;
        break;
      }
      const float2 other = *reinterpret_cast<const float2 *>(sp + xt * kPBytes + (h ^ 1) * kPBox + row * 128);
      __syncwarp();
      if (lane == 0) mbar_arrive(&xdone);
      const float m0 = h == 0 ? m : other.x, l0 = h == 0 ? l : other.y;
      const float m1 = h == 0 ? other.x : m, l1 = h == 0 ? other.y : l;
      const float M = fmaxf(m0, m1);  // finite: key 0 is valid, so half 0 of block 0 has a score
      const float a0 = ex2(m0 - M), a1 = ex2(m1 - M);
      const float inv = 1.0f / (a0 * l0 + a1 * l1);
      const float f0 = a0 * inv, f1 = a1 * inv;

      if (!__all_sync(0xffffffffu, wait_or_abort(&o_full, local & 1, 690, flag))) {
        ok = false;
        break;
      }
      fence_after();
      const bool tma = s.o_tma != 0;
      uint8_t *srow = sp + yt * kPBytes + row * 128;
      if (tma) wait_staged(yt);
      const int r = rt * BM + row;
      __nv_bfloat16 *orow = nullptr;
      if (!tma && r < s.R) {
        const int hq = hk * s.group + r / s.L, pos = r % s.L;
        orow = out + (int64_t)b * s.o_sb + (int64_t)hq * s.o_sh + (int64_t)pos * s.o_sl;
      }
      for (int c = c_lo; c < c_hi; ++c) {
        uint32_t r0[16], r1[16];
        tld16_async(tmem + 256 + lane_off + c * 16, r0);
        tld16_async(tmem + 384 + lane_off + c * 16, r1);
        tld_wait();
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float x0 = fmaf(__uint_as_float(r0[2 * e]), f0, __uint_as_float(r1[2 * e]) * f1);
          const float x1 = fmaf(__uint_as_float(r0[2 * e + 1]), f0, __uint_as_float(r1[2 * e + 1]) * f1);
          __nv_bfloat162 hh = __floats2bfloat162_rn(x0, x1);
          w[e] = *reinterpret_cast<uint32_t *>(&hh);
        }
        if (tma) {
          const int cc = 2 * c;  // 16-byte chunks of 8 columns in the 64-column atom c / 4 (= h)
          *reinterpret_cast<uint4 *>(srow + (cc >> 3) * kPBox + (((uint32_t)(cc & 7) ^ (uint32_t)(row & 7)) << 4)) =
              make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4 *>(srow + ((cc + 1) >> 3) * kPBox +
                                     (((uint32_t)((cc + 1) & 7) ^ (uint32_t)(row & 7)) << 4)) =
              make_uint4(w[4], w[5], w[6], w[7]);
        } else if (orow) {
          const int c0 = c * 16;
          if (c0 + 16 <= s.Dv) {
            uint4 *dst = reinterpret_cast<uint4 *>(orow + c0);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
          } else {
            const __nv_bfloat16 *hv = reinterpret_cast<const __nv_bfloat16 *>(w);
            for (int e = 0; c0 + e < s.Dv; ++e) orow[c0 + e] = hv[e];
          }
        }
      }
      fence_before();
      if (tma) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&o_free);  // O_0 and O_1 are read for this warp's rows and columns
        if (tma && c_lo < c_hi) {
          const int r0 = rt * BM + q4 * 32;
          if (r0 < s.R) {  // a warp's 32 rows lie in one head (checked on the host)
            const int hq = hk * s.group + r0 / s.L, pos = r0 % s.L;
            tma_store(&map_o, sp + yt * kPBytes + h * kPBox + q4 * 32 * 128, h * 64, pos, hq, b);
          }
          bulk_commit();
        }
      }
      __syncwarp();
      if (tma && c_lo < c_hi) staged = yt;
    }
    if (lane == 0) bulk_wait_all();  // this warp's output stores are complete before the CTA exits
    __syncwarp();
  } else if (kSep && warp >= 12) {
    // ---------------- output epilogue (kSep): thread = query row q4·32 + lane, every column
    const int q4 = warp & 3, row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const int nchunk = s.dvp / 16;
    int local = 0;
    for (int item = blockIdx.x; item < s.items && !aborted(flag); item += gridDim.x, ++local) {
      int b, hk, rt;
      item_coords(s, item, b, hk, rt);
      if (!__all_sync(0xffffffffu, wait_or_abort(&lrdy, local & 1, 695, flag))) break;
      if (!__all_sync(0xffffffffu, wait_or_abort(&o_full, local & 1, 696, flag))) break;
      fence_after();
      float m0, l0, m1, l1;
      tld2(tmem + lane_off + 256 + kMLCol, m0, l0);
      tld2(tmem + lane_off + 384 + kMLCol, m1, l1);
      const float M = fmaxf(m0, m1);  // finite: key 0 is valid, so half 0 of block 0 has a score
      const float a0 = ex2(m0 - M), a1 = ex2(m1 - M);
      const float inv = 1.0f / (a0 * l0 + a1 * l1);
      const float f0 = a0 * inv, f1 = a1 * inv;
      uint32_t pk[kSepChunks][8];  // the row as bf16 pairs, so the accumulators are released before the stores
#pragma unroll
      for (int c = 0; c < kSepChunks; ++c) {
        if (c < nchunk) {
          uint32_t r0[16], r1[16];
          tld16_async(tmem + lane_off + 256 + c * 16, r0);
          tld16_async(tmem + lane_off + 384 + c * 16, r1);
          tld_wait();
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float x0 = fmaf(__uint_as_float(r0[2 * e]), f0, __uint_as_float(r1[2 * e]) * f1);
            const float x1 = fmaf(__uint_as_float(r0[2 * e + 1]), f0, __uint_as_float(r1[2 * e + 1]) * f1);
            __nv_bfloat162 hh = __floats2bfloat162_rn(x0, x1);
            pk[c][e] = *reinterpret_cast<uint32_t *>(&hh);
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free);  // O_0, O_1 and (m, l) are read for this warp's rows
      const int r = rt * BM + row;
      if (r < s.R) {
        const int hq = hk * s.group + r / s.L, pos = r % s.L;
        __nv_bfloat16 *orow = out + (int64_t)b * s.o_sb + (int64_t)hq * s.o_sh + (int64_t)pos * s.o_sl;
#pragma unroll
        for (int c = 0; c < kSepChunks; ++c) {
          const int c0 = c * 16;
          if (c < nchunk) {
            uint4 *dst = reinterpret_cast<uint4 *>(orow + c0);
            dst[0] = make_uint4(pk[c][0], pk[c][1], pk[c][2], pk[c][3]);
            // Dv is a multiple of 8: a last chunk holds 8 or 16 columns
            if (c0 + 16 <= s.Dv) dst[1] = make_uint4(pk[c][4], pk[c][5], pk[c][6], pk[c][7]);
          }
        }
      }
    }
  }

  __syncthreads();
  if (aborted(flag) && threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();  // let copies and MMAs in flight drain (bounded)
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  __syncthreads();
  if (warp == 2) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

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

// bf16 tensor (cols, rows, d2, d3) with element strides (row, s2, s3), boxes of 64 × box_rows,
// 128-byte swizzle; the driver's result code, no error recorded.
CUresult encode_map(CUtensorMap *map, const void *base, int64_t cols, int64_t rows, int64_t d2, int64_t d3,
                    int64_t rs, int64_t s2, int64_t s3, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return CUDA_ERROR_NOT_FOUND;
  if (d2 <= 1) s2 = rows * rs;
  if (d3 <= 1) s3 = d2 * s2;
  cuuint64_t dims[4] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)d2, (cuuint64_t)d3};
  cuuint64_t strides[3] = {(cuuint64_t)(rs * 2), (cuuint64_t)(s2 * 2), (cuuint64_t)(s3 * 2)};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

int make_map(CUtensorMap *map, const void *base, int64_t cols, int64_t rows, int64_t d2, int64_t d3, int64_t rs,
             int64_t s2, int64_t s3, int box_rows) {
  DP_REQUIRE(encode_fn() != nullptr, DP_ERR_CUDA, "attention: cuTensorMapEncodeTiled unavailable");
  const CUresult r = encode_map(map, base, cols, rows, d2, d3, rs, s2, s3, box_rows);
  DP_REQUIRE(r == CUDA_SUCCESS, DP_ERR_CUDA,
             "attention: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return DP_OK;
}


template <int BKV>
int stages_for(const Shape &s) {
  const size_t budget = 224 * 1024;  // dynamic shared memory for tiles (the 1 KB alignment slack comes on top)
  const size_t stage = (size_t)(s.nd + s.ndv) * Blk<BKV>::kKVBox;
  const size_t fixed = (size_t)s.q_bytes + 2 * Blk<BKV>::kPBytes;
  if (fixed >= budget) return 0;
  int stages = (int)((budget - fixed) / stage);
  return stages > kMaxStages ? kMaxStages : stages;
}

template <int BKV>
int launch_blocks(const dp_attention_params &p, Shape s, const void *q, const void *k, const void *v, void *o,
                  cudaStream_t stream) {
  const int stages = stages_for<BKV>(s);
  DP_REQUIRE(stages >= 2, DP_ERR_UNSUPPORTED, "attention: head dims too large for the shared-memory ring");
  s.stages = stages;
  s.stage_bytes = (uint32_t)(s.nd + s.ndv) * Blk<BKV>::kKVBox;
  s.kv_blocks = (s.S + BKV - 1) / BKV;
  CUtensorMap mq, mk, mv;
  // Q as (D, group rows R, kv heads, batch): a group's stacked query heads are one row range
  int st = make_map(&mq, q, p.D, s.R, p.heads_kv, p.batch, p.q_sl, p.group * p.q_sh, p.q_sb, BM);
  if (st != DP_OK) return st;
  st = make_map(&mk, k, p.D, p.S, p.heads_kv, p.batch, p.k_ss, p.k_sh, p.k_sb, BKV);
  if (st != DP_OK) return st;
  st = make_map(&mv, v, p.Dv, p.S, p.heads_kv, p.batch, p.v_ss, p.v_sh, p.v_sb, BKV);
  if (st != DP_OK) return st;
  // O as (Dv, L, query heads, batch) in boxes of 64 columns × 32 rows, for 128-key blocks
  // where every warp's 32 rows lie in one head (one query head per item, or L a multiple of 32).
  CUtensorMap mo;
  std::memset(&mo, 0, sizeof(mo));
  s.o_tma = 0;
  if (BKV == 128 && (p.group == 1 || p.L % 32 == 0) &&
      encode_map(&mo, o, p.Dv, p.L, p.heads_kv * p.group, p.batch, p.o_sl, p.o_sh, p.o_sb, 32) == CUDA_SUCCESS)
    s.o_tma = 1;
  const size_t smem = (size_t)s.q_bytes + 2 * Blk<BKV>::kPBytes + (size_t)stages * s.stage_bytes + 1024;
  int dev = 0;
  DP_CHECK_CUDA(cudaGetDevice(&dev));
  static size_t attr_bytes[64] = {};  // one per kernel instantiation (BKV) and device
  DP_REQUIRE(dev >= 0 && dev < 64, DP_ERR_UNSUPPORTED, "attention: device ordinal out of range");
  // 128-key blocks run the split-softmax kernel, 64-key blocks attn_kernel
  int grid = dp::num_sms();
  if (grid > s.items) grid = s.items;
  if constexpr (BKV == 128) {
    // outputs of at most 112 columns: separate epilogue warps
    const bool sep = s.dvp <= kSepMaxDv;
    static size_t attr_sep[64] = {};
    size_t &attr = sep ? attr_sep[dev] : attr_bytes[dev];
    auto kern = sep ? attn_split_kernel<true> : attn_split_kernel<false>;
    if (smem > attr) {
      DP_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      attr = smem;
    }
    dp::launch_k(kern, grid, sep ? kSepThreads : kSplitThreads, smem, stream, mq, mk, mv, mo, s,
                 static_cast<__nv_bfloat16 *>(o));
  } else {
    if (smem > attr_bytes[dev]) {
      DP_CHECK_CUDA(cudaFuncSetAttribute(attn_kernel<BKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      attr_bytes[dev] = smem;
    }
    dp::launch_k(attn_kernel<BKV>, grid, Blk<BKV>::kThreads, smem, stream, mq, mk, mv, s,
                 static_cast<__nv_bfloat16 *>(o));
  }
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

}  // namespace dpk_attn

namespace dp {

int launch_attention(const dp_attention_params &p, const void *q, const void *k, const void *v, void *o,
                     cudaStream_t stream) {
  using namespace dpk_attn;
  DP_REQUIRE(q && k && v && o, DP_ERR_ARG, "attention: null operand");
  DP_REQUIRE(p.dtype == DP_BF16, DP_ERR_UNSUPPORTED, "attention: bf16 operands only");
  DP_REQUIRE(p.batch > 0 && p.heads_kv > 0 && p.group > 0 && p.L > 0 && p.S > 0 && p.D > 0 && p.Dv > 0,
             DP_ERR_SHAPE, "attention: sizes must be positive");
  DP_REQUIRE(p.D <= 256 && p.Dv <= 256 && p.D % 8 == 0 && p.Dv % 8 == 0, DP_ERR_UNSUPPORTED,
             "attention: head dims must be multiples of 8, at most 256");
  const int64_t strides[] = {p.q_sb, p.q_sh, p.q_sl, p.k_sb, p.k_sh, p.k_ss,
                             p.v_sb, p.v_sh, p.v_ss, p.o_sb, p.o_sh, p.o_sl};
  for (int64_t x : strides)
    DP_REQUIRE(x >= 0 && x % 8 == 0, DP_ERR_UNSUPPORTED, "attention: strides must be multiples of 8 elements");
  auto al = [](const void *ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; };
  DP_REQUIRE(al(q) && al(k) && al(v) && al(o), DP_ERR_UNSUPPORTED, "attention: 16-byte aligned bases needed");
  DP_REQUIRE(p.group == 1 || (p.q_sh == p.L * p.q_sl && p.o_sh == p.L * p.o_sl), DP_ERR_UNSUPPORTED,
             "attention: a group's query heads must be stacked rows");
  DP_REQUIRE(p.group * p.L < (1ll << 30) && p.S < (1ll << 30), DP_ERR_UNSUPPORTED, "attention: too many rows");
  Shape s{};
  s.L = (int)p.L;
  s.R = (int)(p.group * p.L);
  s.S = (int)p.S;
  s.D = (int)p.D;
  s.Dv = (int)p.Dv;
  s.nd = (int)((p.D + 63) / 64);
  s.ndv = (int)((p.Dv + 63) / 64);
  s.ks = (int)((p.D + 15) / 16);
  s.dvp = (int)((p.Dv + 15) / 16 * 16);
  s.q_bytes = (uint32_t)s.nd * kQBox;
  s.tiles_r = (s.R + BM - 1) / BM;
  s.heads_kv = (int)p.heads_kv;
  s.group = (int)p.group;
  const int64_t items = p.batch * p.heads_kv * s.tiles_r;
  DP_REQUIRE(items < (1ll << 31), DP_ERR_UNSUPPORTED, "attention: too many work items");
  s.items = (int)items;
  s.scale_log2 = p.scale * 1.4426950408889634f;
  // The kernel forms score · scale − max by one FMA, where a masked key's
  // −∞ score times a zero scale would give NaN: a zero scale runs as 1e-30
  // (every valid key's exponent is then 0 to within rounding, as for 0).
  if (s.scale_log2 == 0.0f) s.scale_log2 = 1e-30f;
  s.o_sb = p.o_sb;
  s.o_sh = p.o_sh;
  s.o_sl = p.o_sl;
  // 128-key blocks when the score and output columns fit TMEM (2·128 + dvp ≤ 512) and two stages fit
  if (p.D <= 128 && p.Dv <= 128 && stages_for<128>(s) >= 2)
    return launch_blocks<128>(p, s, q, k, v, o, stream);
  return launch_blocks<64>(p, s, q, k, v, o, stream);
}

}  // namespace dp

extern "C" int dp_attention(const dp_attention_params *p, const void *q, const void *k, const void *v, void *o,
                            void *stream) {
  if (!p) return dp::set_error(DP_ERR_ARG, "dp_attention: null params");
  return dp::launch_attention(*p, q, k, v, o, dp::as_stream(stream));
}
