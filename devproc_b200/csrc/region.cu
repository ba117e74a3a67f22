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
// with rank 1 and unit/zero strides each thread moves four consecutive
// elements with vector loads.
#include "dp_common.cuh"

namespace dpk_region {

constexpr int E = 4;  // elements per thread
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

// FAST: rank 1, every stride 0 or 1.
template <bool FAST>
__global__ void __launch_bounds__(kThreads) region_kernel(const dp_region_desc d, Ops c, int64_t total) {
  const int64_t base = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * E;
  const int64_t gstride = (int64_t)gridDim.x * blockDim.x * E;
  for (int64_t i0 = base; i0 < total; i0 += gstride) {
    int64_t coord[E][DP_REGION_MAX_RANK];
    if (!FAST) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        int64_t idx = i0 + e;
        for (int k = d.rank - 1; k >= 0; --k) {
          coord[e][k] = idx % d.shape[k];
          idx /= d.shape[k];
        }
      }
    }
    const int n_live = (total - i0) < E ? (int)(total - i0) : E;
    float r[DP_REGION_MAX_REGS][E];
    for (int pc = 0; pc < d.n_instr; ++pc) {
      const uint32_t ins = d.instr[pc];
      const int op = ins & 0xff, dst = (ins >> 8) & 0xff, a = (ins >> 16) & 0xff, b = (ins >> 24) & 0xff;
      if (op == DP_OP_LOAD || op == DP_OP_STORE) {
        const int operand = a;
        void *ptr = const_cast<void *>(c.p[operand]);
        const int dt = d.dtype[operand];
#pragma unroll
        for (int e = 0; e < E; ++e) {
          if (e >= n_live) break;
          int64_t off = 0;
          if (FAST) {
            off = d.stride[operand][0] * (i0 + e);
          } else {
            for (int k = 0; k < d.rank; ++k) off += coord[e][k] * d.stride[operand][k];
          }
          if (op == DP_OP_LOAD)
            r[dst][e] = load_as_f32(ptr, off, dt);
          else
            store_from_f32(ptr, off, dt, r[b][e]);
        }
      } else if (op == DP_OP_CONST) {
#pragma unroll
        for (int e = 0; e < E; ++e) r[dst][e] = d.consts[a];
      } else if (op == DP_OP_CHANSEL) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          int64_t cc;
          if (FAST) {
            cc = (i0 + e) % d.shape[0];
          } else {
            cc = coord[e][b];
          }
          r[dst][e] = d.consts[a + (int)cc];
        }
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


// Tiled transpose for pure copies whose output's innermost dim is strided in
// the input (e.g. a [.., S, D] → [.., D, S] relayout): 32×32 tiles through
// shared memory, reads coalesced along the input's unit-stride dim, writes
// coalesced along the output's innermost dim.  Remaining dims are decomposed
// from blockIdx.z once per block.
struct TDims {
  int rank;  // of the collapsed iteration space
  int jdim;  // dim with unit input stride
  int64_t shape[DP_REGION_MAX_RANK];
  int64_t in_stride[DP_REGION_MAX_RANK];
  int64_t out_stride[DP_REGION_MAX_RANK];
};

template <typename T>
__global__ void __launch_bounds__(256) transpose_copy_kernel(TDims d, const T *__restrict__ in, T *__restrict__ out) {
  __shared__ T tile[32][33];
  const int last = d.rank - 1;
  const int64_t j0 = (int64_t)blockIdx.y * 32, l0 = (int64_t)blockIdx.x * 32;
  // offsets of the other dims
  int64_t z = blockIdx.z, in_off = 0, out_off = 0;
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
        } else if (op >= DP_OP_NEG && op <= DP_OP_MOV) {
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
          case 1: transpose_copy_kernel<uint8_t><<<grid, 256, 0, s>>>(t, (const uint8_t *)ops[0], (uint8_t *)ops[1]); break;
          case 2: transpose_copy_kernel<uint16_t><<<grid, 256, 0, s>>>(t, (const uint16_t *)ops[0], (uint16_t *)ops[1]); break;
          case 4: transpose_copy_kernel<uint32_t><<<grid, 256, 0, s>>>(t, (const uint32_t *)ops[0], (uint32_t *)ops[1]); break;
          default: transpose_copy_kernel<uint64_t><<<grid, 256, 0, s>>>(t, (const uint64_t *)ops[0], (uint64_t *)ops[1]); break;
        }
        DP_CHECK_CUDA(cudaGetLastError());
        return DP_OK;
      }
    }
  }
  bool fast = d.rank == 1;
  for (int i = 0; i < n_ops && fast; ++i) fast = d.stride[i][0] == 0 || d.stride[i][0] == 1;
  Ops c{};
  for (int i = 0; i < n_ops; ++i) c.p[i] = ops[i];
  const int64_t groups = (total + E - 1) / E;
  int64_t blocks = (groups + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  if (fast)
    region_kernel<true><<<(int)blocks, kThreads, 0, s>>>(d, c, total);
  else
    region_kernel<false><<<(int)blocks, kThreads, 0, s>>>(d, c, total);
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

}  // namespace dp

extern "C" int dp_region(const dp_region_desc *d, const void *const *operands, void *stream) {
  if (!d) return dp::set_error(DP_ERR_ARG, "dp_region: null desc");
  return dp::launch_region(*d, operands, dp::as_stream(stream));
}
