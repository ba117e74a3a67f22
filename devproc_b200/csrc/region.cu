// Elementwise region kernel: one launch runs a whole fused chain of
// elementwise IR ops (casts, normalise, activations, broadcast arithmetic,
// transposes) as a small register program per element.
//
// Replaces the reference's one-launch-per-op elementwise templates
// (src/devproc/backend/triton/templates/elementwise.py:11-184), whose tail
// mask ignored the block offset (:20-22), and its torch fallback for
// transpose (src/devproc/backend/triton/ops.py:418-420).
//
// The iteration space is the region's output shape; every operand carries
// per-dim element strides (0 = broadcast, permuted strides = transpose), so
// a transpose is just a strided load.  The host collapses contiguous dims;
// each thread then works on runs of up to 8 elements along the innermost
// dim, with 16-byte loads and stores where the run is unit-stride.
#include <type_traits>

#include "dp_common.cuh"

namespace dpk_region {

constexpr int kThreads = 256;

// Operand pointers, passed to the kernel by value.
struct Ops {
  const void *p[DP_REGION_MAX_OPERANDS];
};

__device__ __forceinline__ float apply_unary(int op, float x) {
  switch (op) {
    case DP_OP_NEG: return -x;
    case DP_OP_ABS: return fabsf(x);
    case DP_OP_RELU: return x > 0.0f ? x : (isnan(x) ? x : 0.0f);
    case DP_OP_SIGMOID: return 1.0f / (1.0f + expf(-x));
    case DP_OP_TANH: return tanhf(x);
    case DP_OP_EXP: return expf(x);
    case DP_OP_GELU_ERF: return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
    case DP_OP_GELU_TANH: {
      const float k0 = 0.7978845608028654f, k1 = 0.044715f;
      return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
    }
    case DP_OP_SILU: return x / (1.0f + expf(-x));
    case DP_OP_TF32: return __uint_as_float(__float_as_uint(x) & 0xffffe000u);
    default: return x;  // MOV
  }
}

__device__ __forceinline__ float apply_binary(int op, float a, float b) {
  switch (op) {
    case DP_OP_ADD: return a + b;
    case DP_OP_SUB: return a - b;
    case DP_OP_MUL: return a * b;
    case DP_OP_DIV: return a / b;
    case DP_OP_MAX: return (a > b || isnan(a)) ? a : b;
    default: return (a < b || isnan(a)) ? a : b;  // MIN
  }
}

// ---------------------------------------------------------------------------
// Iteration geometry.  The collapsed dims are right-aligned into kR slots
// (leading slots have extent 1), so every coordinate loop is unrolled with
// static indices.  One work item is a run of E consecutive elements along the
// innermost dim (E divides its extent); its coordinates come from one mixed-
// radix decomposition of the item index with magic-number division
// (FastDiv, exact for indices below 2^31), then each operand's offset is one
// dot product.
constexpr int kR = DP_REGION_MAX_RANK;

struct Geom {
  int64_t items;                                // work items (runs of E elements)
  int64_t off[DP_REGION_MAX_OPERANDS];          // element offset of each operand's first element
  int64_t ext[kR];                              // extents; ext[kR-1] counted in runs
  int64_t stride[DP_REGION_MAX_OPERANDS][kR];   // element strides, right-aligned
  FastDiv fd[kR];                               // divisors of ext (32-bit path)
  int chan_slot[DP_REGION_MAX_INSTR];           // right-aligned dim of each CHANSEL
};

// E elements of one operand: a 16-byte-or-narrower vector when the run is
// unit-stride and aligned, one broadcast load when the stride is 0.
template <int E>
__device__ __forceinline__ void load_run(const void *ptr, int64_t off, int64_t st, int dt, float (&v)[E]) {
  if (st == 0) {
    const float x = load_as_f32(ptr, off, dt);
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = x;
    return;
  }
  if (st == 1) {
    const int es = dt == DP_BF16 ? 2 : 4;  // the vector paths below take bf16 and f32
    const uintptr_t a = reinterpret_cast<uintptr_t>(ptr) + (uintptr_t)(off * es);
    if (dt == DP_BF16 && E >= 2 && a % (2 * E < 16 ? 2 * E : 16) == 0) {
      const __nv_bfloat162 *q = reinterpret_cast<const __nv_bfloat162 *>(a);
      if constexpr (E == 8) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(a));
        q = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
        for (int e = 0; e < E / 2; ++e) {
          const float2 f = __bfloat1622float2(q[e]);
          v[2 * e] = f.x;
          v[2 * e + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < E / 2; ++e) {
          const float2 f = __bfloat1622float2(q[e]);
          v[2 * e] = f.x;
          v[2 * e + 1] = f.y;
        }
      }
      return;
    }
    if (dt == DP_F32 && E >= 4 && a % 16 == 0) {
#pragma unroll
      for (int e = 0; e < E; e += 4) {
        const float4 f = __ldg(reinterpret_cast<const float4 *>(a) + e / 4);
        v[e] = f.x;
        v[e + 1] = f.y;
        v[e + 2] = f.z;
        v[e + 3] = f.w;
      }
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = load_as_f32(ptr, off + e * st, dt);
}

template <int E>
__device__ __forceinline__ void store_run(void *ptr, int64_t off, int64_t st, int dt, const float (&v)[E]) {
  if (st == 1) {
    const int es = dt == DP_BF16 ? 2 : 4;  // the vector paths below take bf16 and f32
    const uintptr_t a = reinterpret_cast<uintptr_t>(ptr) + (uintptr_t)(off * es);
    if (dt == DP_BF16 && E >= 2 && a % (2 * E < 16 ? 2 * E : 16) == 0) {
      __nv_bfloat162 h[E / 2 > 0 ? E / 2 : 1];
#pragma unroll
      for (int e = 0; e < E / 2; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
      if constexpr (E == 8) {
        *reinterpret_cast<uint4 *>(a) = *reinterpret_cast<const uint4 *>(h);
      } else {
#pragma unroll
        for (int e = 0; e < E / 2; ++e) reinterpret_cast<__nv_bfloat162 *>(a)[e] = h[e];
      }
      return;
    }
    if (dt == DP_F32 && E >= 4 && a % 16 == 0) {
#pragma unroll
      for (int e = 0; e < E; e += 4)
        reinterpret_cast<float4 *>(a)[e / 4] = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) store_from_f32(ptr, off + e * st, dt, v[e]);
}

// Register-program interpreter over runs of E elements.  WIDE: 64-bit
// item decomposition (more than 2^31 items).
template <int E, bool WIDE>
__global__ void __launch_bounds__(kThreads) region_kernel(const dp_region_desc d, Ops c, const Geom g) {
  dp::pdl_trigger();
  dp::pdl_wait();
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < g.items; t += nthreads) {
    int64_t coord[kR];
    if constexpr (WIDE) {
      int64_t rest = t;
#pragma unroll
      for (int k = kR - 1; k >= 0; --k) {
        const int64_t q = rest / g.ext[k];
        coord[k] = rest - q * g.ext[k];
        rest = q;
      }
    } else {
      uint32_t rest = (uint32_t)t;
#pragma unroll
      for (int k = kR - 1; k >= 0; --k) {
        const uint32_t q = g.fd[k].d == 1 ? rest : fdiv(rest, g.fd[k]);
        coord[k] = (int64_t)(rest - q * g.fd[k].d);
        rest = q;
      }
    }
    coord[kR - 1] *= E;  // element index of the run's first element
    float r[DP_REGION_MAX_REGS][E];
    for (int pc = 0; pc < d.n_instr; ++pc) {
      const uint32_t ins = d.instr[pc];
      const int op = ins & 0xff, dst = (ins >> 8) & 0xff, a = (ins >> 16) & 0xff, b = (ins >> 24) & 0xff;
      if (op == DP_OP_LOAD || op == DP_OP_STORE) {
        int64_t off = g.off[a];
#pragma unroll
        for (int k = 0; k < kR; ++k) off += coord[k] * g.stride[a][k];
        if (op == DP_OP_LOAD)
          load_run<E>(c.p[a], off, g.stride[a][kR - 1], d.dtype[a], r[dst]);
        else
          store_run<E>(const_cast<void *>(c.p[a]), off, g.stride[a][kR - 1], d.dtype[a], r[b]);
      } else if (op == DP_OP_CONST) {
#pragma unroll
        for (int e = 0; e < E; ++e) r[dst][e] = d.consts[a];
      } else if (op == DP_OP_CHANSEL) {
        const int slot = g.chan_slot[pc];
        int64_t cc = 0;
#pragma unroll
        for (int k = 0; k < kR; ++k)
          if (k == slot) cc = coord[k];
#pragma unroll
        for (int e = 0; e < E; ++e) r[dst][e] = d.consts[a + (int)(slot == kR - 1 ? cc + e : cc)];
      } else if (op >= DP_OP_ADD && op <= DP_OP_MIN) {
#pragma unroll
        for (int e = 0; e < E; ++e) r[dst][e] = apply_binary(op, r[a][e], r[b][e]);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) r[dst][e] = apply_unary(op, r[a][e]);
      }
    }
  }
}

// Pure copies between operands of one dtype move raw elements (no float
// round trip, so 32/64-bit integers survive), E per work item.
template <typename T, int E, bool WIDE>
__global__ void __launch_bounds__(kThreads) copy_kernel(const T *__restrict__ in, T *__restrict__ out, const Geom g) {
  dp::pdl_trigger();
  dp::pdl_wait();
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < g.items; t += nthreads) {
    int64_t coord[kR];
    if constexpr (WIDE) {
      int64_t rest = t;
#pragma unroll
      for (int k = kR - 1; k >= 0; --k) {
        const int64_t q = rest / g.ext[k];
        coord[k] = rest - q * g.ext[k];
        rest = q;
      }
    } else {
      uint32_t rest = (uint32_t)t;
#pragma unroll
      for (int k = kR - 1; k >= 0; --k) {
        const uint32_t q = g.fd[k].d == 1 ? rest : fdiv(rest, g.fd[k]);
        coord[k] = (int64_t)(rest - q * g.fd[k].d);
        rest = q;
      }
    }
    coord[kR - 1] *= E;
    int64_t io = g.off[0], oo = g.off[1];
#pragma unroll
    for (int k = 0; k < kR; ++k) {
      io += coord[k] * g.stride[0][k];
      oo += coord[k] * g.stride[1][k];
    }
    const int64_t is = g.stride[0][kR - 1], os = g.stride[1][kR - 1];
    constexpr int kRunBytes = (int)sizeof(T) * E;
    if constexpr (kRunBytes == 4 || kRunBytes == 8 || kRunBytes == 16) {
      using V = std::conditional_t<kRunBytes == 16, uint4, std::conditional_t<kRunBytes == 8, uint2, uint32_t>>;
      const T *src = in + io;
      T *dst = out + oo;
      if (is == 1 && os == 1 && reinterpret_cast<uintptr_t>(src) % kRunBytes == 0 &&
          reinterpret_cast<uintptr_t>(dst) % kRunBytes == 0) {
        *reinterpret_cast<V *>(dst) = __ldg(reinterpret_cast<const V *>(src));
        continue;
      }
    }
    T v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = in[io + e * is];
#pragma unroll
    for (int e = 0; e < E; ++e) out[oo + e * os] = v[e];
  }
}

// Tiled transpose for pure copies whose output's innermost dim is strided in
// the input (e.g. a [.., S, D] → [.., D, S] relayout): 32×32 tiles through
// shared memory, reads coalesced along the input's unit-stride dim, writes
// coalesced along the output's innermost dim.  Remaining dims are decomposed
// from blockIdx.z once per block.
struct TDims {
  int rank;  // of the collapsed iteration space
  int jdim;  // dim with unit input stride
  int64_t in_base, out_base;  // element offsets of the first elements
  int64_t shape[DP_REGION_MAX_RANK];
  int64_t in_stride[DP_REGION_MAX_RANK];
  int64_t out_stride[DP_REGION_MAX_RANK];
};

template <typename T>
__global__ void __launch_bounds__(256) transpose_copy_kernel(TDims d, const T *__restrict__ in, T *__restrict__ out) {
  dp::pdl_trigger();
  dp::pdl_wait();
  __shared__ T tile[32][33];
  const int last = d.rank - 1;
  const int64_t j0 = (int64_t)blockIdx.y * 32, l0 = (int64_t)blockIdx.x * 32;
  // offsets of the other dims
  int64_t z = blockIdx.z, in_off = d.in_base, out_off = d.out_base;
  for (int k = last; k >= 0; --k) {
    if (k == last || k == d.jdim) continue;
    const int64_t c = z % d.shape[k];
    z /= d.shape[k];
    in_off += c * d.in_stride[k];
    out_off += c * d.out_stride[k];
  }
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 × 8
  // read: lanes walk j (unit stride in the input)
  for (int r = ty; r < 32; r += 8) {
    const int64_t j = j0 + tx, l = l0 + r;
    if (j < d.shape[d.jdim] && l < d.shape[last]) tile[r][tx] = in[in_off + j + l * d.in_stride[last]];
  }
  __syncthreads();
  // write: lanes walk the output's innermost dim
  for (int r = ty; r < 32; r += 8) {
    const int64_t j = j0 + r, l = l0 + tx;
    if (j < d.shape[d.jdim] && l < d.shape[last]) out[out_off + j * d.out_stride[d.jdim] + l] = tile[tx][r];
  }
}

}  // namespace dpk_region

namespace dp {

int launch_region(const dp_region_desc &d, const void *const *ops, cudaStream_t s) {
  using namespace dpk_region;
  DP_REQUIRE(ops != nullptr, DP_ERR_ARG, "region: null operand array");
  DP_REQUIRE(d.rank >= 1 && d.rank <= DP_REGION_MAX_RANK, DP_ERR_ARG, "region: rank out of range");
  DP_REQUIRE(d.n_in >= 0 && d.n_out >= 1 && d.n_in + d.n_out <= DP_REGION_MAX_OPERANDS, DP_ERR_ARG,
             "region: operand count out of range");
  DP_REQUIRE(d.n_instr >= 1 && d.n_instr <= DP_REGION_MAX_INSTR, DP_ERR_ARG, "region: instruction count");
  int64_t total = 1;
  for (int k = 0; k < d.rank; ++k) {
    DP_REQUIRE(d.shape[k] > 0, DP_ERR_SHAPE, "region: shape must be positive");
    total *= d.shape[k];
  }
  const int n_ops = d.n_in + d.n_out;
  for (int i = 0; i < n_ops; ++i) {
    DP_REQUIRE(ops[i] != nullptr, DP_ERR_ARG, "region: null operand " + std::to_string(i));
    DP_REQUIRE(dtype_bytes(d.dtype[i]) > 0, DP_ERR_ARG, "region: bad dtype of operand " + std::to_string(i));
    DP_REQUIRE(d.offset[i] >= 0, DP_ERR_ARG, "region: negative offset of operand " + std::to_string(i));
  }
  // Validate the program on the host so the kernel never indexes out of range.
  for (int pc = 0; pc < d.n_instr; ++pc) {
    const uint32_t ins = d.instr[pc];
    const int op = ins & 0xff, dst = (ins >> 8) & 0xff, a = (ins >> 16) & 0xff, b = (ins >> 24) & 0xff;
    const std::string where = "region: instruction " + std::to_string(pc);
    switch (op) {
      case DP_OP_LOAD:
        DP_REQUIRE(a < d.n_in && dst < DP_REGION_MAX_REGS, DP_ERR_ARG, where + " bad load");
        break;
      case DP_OP_STORE:
        DP_REQUIRE(a >= d.n_in && a < n_ops && b < DP_REGION_MAX_REGS, DP_ERR_ARG, where + " bad store");
        break;
      case DP_OP_CONST:
        DP_REQUIRE(a < DP_REGION_MAX_CONST && dst < DP_REGION_MAX_REGS, DP_ERR_ARG, where + " bad const");
        break;
      case DP_OP_CHANSEL:
        DP_REQUIRE(b < d.rank && dst < DP_REGION_MAX_REGS, DP_ERR_ARG, where + " bad chansel dim");
        DP_REQUIRE(a + d.shape[d.rank == 1 ? 0 : b] <= DP_REGION_MAX_CONST, DP_ERR_ARG, where + " chansel consts");
        break;
      default:
        if (op >= DP_OP_ADD && op <= DP_OP_MIN) {
          DP_REQUIRE(dst < DP_REGION_MAX_REGS && a < DP_REGION_MAX_REGS && b < DP_REGION_MAX_REGS, DP_ERR_ARG,
                     where + " bad registers");
        } else if (op >= DP_OP_NEG && op <= DP_OP_TF32) {
          DP_REQUIRE(dst < DP_REGION_MAX_REGS && a < DP_REGION_MAX_REGS, DP_ERR_ARG, where + " bad registers");
        } else {
          return set_error(DP_ERR_ARG, where + " unknown opcode " + std::to_string(op));
        }
    }
  }
  // Pure relayout copies (one load, one store, same element size) whose
  // innermost output dim is strided in the input go to the tiled transpose.
  if (d.n_in == 1 && d.n_out == 1 && d.n_instr == 2 && d.rank >= 2 &&
      dtype_bytes(d.dtype[0]) == dtype_bytes(d.dtype[1]) && d.dtype[0] == d.dtype[1] &&
      (d.instr[0] & 0xff) == DP_OP_LOAD && (d.instr[1] & 0xff) == DP_OP_STORE &&
      d.stride[1][d.rank - 1] == 1 && d.stride[0][d.rank - 1] != 1) {
    int jdim = -1;
    for (int k = 0; k < d.rank - 1; ++k)
      if (d.stride[0][k] == 1) jdim = k;
    if (jdim >= 0) {
      TDims t;
      t.rank = d.rank;
      t.jdim = jdim;
      t.in_base = d.offset[0];
      t.out_base = d.offset[1];
      int64_t zcount = 1;
      for (int k = 0; k < d.rank; ++k) {
        t.shape[k] = d.shape[k];
        t.in_stride[k] = d.stride[0][k];
        t.out_stride[k] = d.stride[1][k];
        if (k != jdim && k != d.rank - 1) zcount *= d.shape[k];
      }
      const int64_t gx = (d.shape[d.rank - 1] + 31) / 32, gy = (d.shape[jdim] + 31) / 32;
      if (gx < (1ll << 31) && gy < 65536 && zcount < 65536) {
        dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)zcount);
        switch (dtype_bytes(d.dtype[0])) {
          case 1: dp::launch_k(transpose_copy_kernel<uint8_t>, grid, 256, 0, s, t, (const uint8_t *)ops[0], (uint8_t *)ops[1]); break;
          case 2: dp::launch_k(transpose_copy_kernel<uint16_t>, grid, 256, 0, s, t, (const uint16_t *)ops[0], (uint16_t *)ops[1]); break;
          case 4: dp::launch_k(transpose_copy_kernel<uint32_t>, grid, 256, 0, s, t, (const uint32_t *)ops[0], (uint32_t *)ops[1]); break;
          default: dp::launch_k(transpose_copy_kernel<uint64_t>, grid, 256, 0, s, t, (const uint64_t *)ops[0], (uint64_t *)ops[1]); break;
        }
        DP_CHECK_CUDA(cudaGetLastError());
        return DP_OK;
      }
    }
  }
  // Runs of E elements along the innermost dim.
  const int64_t inner = d.shape[d.rank - 1];
  const int E = inner % 8 == 0 ? 8 : inner % 4 == 0 ? 4 : inner % 2 == 0 ? 2 : 1;
  Geom g{};
  const int lead = kR - d.rank;
  for (int k = 0; k < kR; ++k) {
    g.ext[k] = k < lead ? 1 : d.shape[k - lead];
    for (int i = 0; i < n_ops; ++i) g.stride[i][k] = k < lead ? 0 : d.stride[i][k - lead];
  }
  g.ext[kR - 1] /= E;
  g.items = total / E;
  for (int i = 0; i < n_ops; ++i) g.off[i] = d.offset[i];
  const bool wide = g.items >= (1ll << 31);
  for (int k = 0; k < kR; ++k) {
    g.fd[k] = make_fastdiv((uint32_t)(wide ? 1 : g.ext[k]));
  }
  for (int pc = 0; pc < d.n_instr; ++pc)
    g.chan_slot[pc] = (d.instr[pc] & 0xff) == DP_OP_CHANSEL ? (int)((d.instr[pc] >> 24) & 0xff) + lead : 0;
  int64_t blocks = (g.items + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  const bool pure_copy = d.n_in == 1 && d.n_out == 1 && d.n_instr == 2 && d.dtype[0] == d.dtype[1] &&
                         (d.instr[0] & 0xff) == DP_OP_LOAD && (d.instr[1] & 0xff) == DP_OP_STORE;
  const dim3 grid((unsigned)blocks), block(kThreads);
#define DP_REGION_LAUNCH(EE)                                                                          \
  do {                                                                                                \
    if (pure_copy) {                                                                                  \
      switch (dtype_bytes(d.dtype[0])) {                                                              \
        case 1:                                                                                       \
          if (wide) dp::launch_k(copy_kernel<uint8_t, EE, true>, grid, block, 0, s, (const uint8_t *)ops[0], (uint8_t *)ops[1], g); \
          else dp::launch_k(copy_kernel<uint8_t, EE, false>, grid, block, 0, s, (const uint8_t *)ops[0], (uint8_t *)ops[1], g);    \
          break;                                                                                      \
        case 2:                                                                                       \
          if (wide) dp::launch_k(copy_kernel<uint16_t, EE, true>, grid, block, 0, s, (const uint16_t *)ops[0], (uint16_t *)ops[1], g); \
          else dp::launch_k(copy_kernel<uint16_t, EE, false>, grid, block, 0, s, (const uint16_t *)ops[0], (uint16_t *)ops[1], g);    \
          break;                                                                                      \
        case 4:                                                                                       \
          if (wide) dp::launch_k(copy_kernel<uint32_t, EE, true>, grid, block, 0, s, (const uint32_t *)ops[0], (uint32_t *)ops[1], g); \
          else dp::launch_k(copy_kernel<uint32_t, EE, false>, grid, block, 0, s, (const uint32_t *)ops[0], (uint32_t *)ops[1], g);    \
          break;                                                                                      \
        default:                                                                                      \
          if (wide) dp::launch_k(copy_kernel<uint64_t, EE, true>, grid, block, 0, s, (const uint64_t *)ops[0], (uint64_t *)ops[1], g); \
          else dp::launch_k(copy_kernel<uint64_t, EE, false>, grid, block, 0, s, (const uint64_t *)ops[0], (uint64_t *)ops[1], g);    \
          break;                                                                                      \
      }                                                                                               \
    } else if (wide) {                                                                                \
      dp::launch_k(region_kernel<EE, true>, grid, block, 0, s, d, c, g);                                        \
    } else {                                                                                          \
      dp::launch_k(region_kernel<EE, false>, grid, block, 0, s, d, c, g);                                       \
    }                                                                                                 \
  } while (0)
  Ops c{};
  for (int i = 0; i < n_ops; ++i) c.p[i] = ops[i];
  switch (E) {
    case 8: DP_REGION_LAUNCH(8); break;
    case 4: DP_REGION_LAUNCH(4); break;
    case 2: DP_REGION_LAUNCH(2); break;
    default: DP_REGION_LAUNCH(1); break;
  }
#undef DP_REGION_LAUNCH
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

}  // namespace dp

extern "C" int dp_region(const dp_region_desc *d, const void *const *operands, void *stream) {
  if (!d) return dp::set_error(DP_ERR_ARG, "dp_region: null desc");
  return dp::launch_region(*d, operands, dp::as_stream(stream));
}
