/*
 * devproc_b200.h — C ABI of the DevProc B200 execution backend.
 *
 * Plain pointers, sizes and POD parameter blocks; no torch or C++ types.
 * Every function returns an int status (DP_OK == 0); on failure the calling
 * thread's last error text is available through dp_last_error().  No call
 * falls back to another implementation: an unsupported case is an error.
 *
 * Stream arguments are cudaStream_t passed as void* (NULL = legacy default
 * stream).  Kernels are enqueued asynchronously; nothing here synchronises
 * except dp_device_error() and dp_program_create().
 *
 * Reference interfaces replaced (paths inside the DevProc project):
 *   dp_program_*     ← TritonCompiledProgram.run/_run_jit_with_ir,
 *                      src/devproc/backend/triton/compiler.py:54-68, 206-250,
 *                      and the ctypes launcher that never ran,
 *                      src/devproc/backend/triton/runtime/kernel_launcher.py:59-273
 *   dp_preproc       ← handle_resize / handle_normalize / handle_to /
 *                      handle_transpose, src/devproc/backend/triton/ops.py:21-53,
 *                      320-432, templates/elementwise.py:11-31, 80-101
 *   dp_rowreduce     ← launch_argmax / launch_softmax / launch_reduce_sum,
 *                      src/devproc/backend/triton/templates/reduce.py:151-214
 *   dp_gemm          ← launch_matmul / launch_linear,
 *                      src/devproc/backend/triton/templates/matmul.py:230-296
 *   dp_region        ← launch_relu / launch_sigmoid / launch_add / launch_to_dtype,
 *                      src/devproc/backend/triton/templates/elementwise.py:132-184
 *   dp_embedding     ← (no reference kernel; FX "embedding" was unsupported,
 *                      src/devproc/ir/fx_converter.py:197-199)
 */
#ifndef DEVPROC_B200_H
#define DEVPROC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DP_ABI_VERSION 1

/* ---- status codes ---------------------------------------------------- */
enum {
  DP_OK = 0,
  DP_ERR_ARG = 1,         /* null pointer, bad enum, bad size            */
  DP_ERR_SHAPE = 2,       /* shape / dtype / byte-size mismatch          */
  DP_ERR_CUDA = 3,        /* a CUDA runtime or driver call failed        */
  DP_ERR_UNSUPPORTED = 4, /* valid request this backend does not handle  */
  DP_ERR_PLAN = 5,        /* malformed program plan                      */
  DP_ERR_STATE = 6,       /* e.g. running a program with unbound slots   */
  DP_ERR_DEVICE = 7       /* a kernel reported an error through the device error word */
};

/* ---- element types ---------------------------------------------------- */
enum {
  DP_U8 = 0, DP_I8 = 1, DP_I16 = 2, DP_I32 = 3, DP_I64 = 4,
  DP_F16 = 5, DP_BF16 = 6, DP_F32 = 7, DP_F64 = 8, DP_BOOL = 9,
  /* GEMM operands only: fp32 in memory, multiplied as TF32 on the tensor
   * cores (the low 13 mantissa bits are not used).  Split x = hi + lo
   * operands give fp32-level products (3xTF32). */
  DP_TF32 = 10
};

/* ---- device error word codes (read with dp_device_error) -------------- */
enum {
  DP_DEVERR_NONE = 0,
  DP_DEVERR_INDEX = 1,    /* embedding id out of range (row written as zeros) */
  DP_DEVERR_TIMEOUT = 2   /* a bounded wait inside a kernel gave up            */
};

/* ---- library ----------------------------------------------------------- */
int dp_version(void);                         /* returns DP_ABI_VERSION*10000 + minor */
int dp_last_error(char *buf, size_t buf_len); /* copies this thread's last error text */
int dp_device_init(int device);               /* sets the device, checks it is sm_100 */
/* Reads and clears the device error word of the current device (synchronises
 * the device).  *code receives a DP_DEVERR_* value, *info the first bad index
 * or wait site recorded. */
int dp_device_error(int *code, int64_t *info);
/* The DP_DEVERR_* code a kernel recorded on ``device`` since the word was last
 * cleared, read from a pinned host mirror that dp_device_init sets up: no CUDA
 * call and no synchronisation, so call it after synchronising the stream the
 * work ran on; then dp_device_error for the site and to clear.  The reference
 * reported no kernel failure at all: it warned and skipped ops
 * (src/devproc/backend/triton/compiler.py:70-74, 302-304, 343-346). */
int dp_device_error_pending(int device, int *code);
/* Wall-time limit of the bounded waits of the row-reduction and preprocessing
 * kernels on ``device`` (0 restores the default, 2 s).  Waits that drain copies
 * in flight before a CTA exits keep their own fixed limit.  No reference
 * counterpart (the reference has no device-side waits). */
int dp_set_wait_limit(int device, uint64_t limit_ns);
/* Failure-detection test switch, off by default: while enabled, the staged
 * fp32 softmax / RMSNorm / LayerNorm kernel on ``device`` arms its row
 * barriers but issues no copy, so its waits can only end by their limit and
 * the kernel reports DP_DEVERR_TIMEOUT (site 700) and returns.  No reference
 * counterpart. */
int dp_test_withhold_copies(int device, int enable);

/* ---- fused preprocessing region ------------------------------------------
 * out[b, c, y, x] (or out[b, y, x, c]) =
 *     cast((bilinear(in)[b, y, x, c] - mean[c]) / std[c])
 * bilinear = align_corners=False, computed in fp32 with no intermediate
 * rounding; identical sizes copy exactly.  Input uint8 / fp32 / bf16 / fp16,
 * layout NHWC or NCHW; output fp32 / bf16 / fp16, layout NCHW or NHWC. */
enum { DP_LAYOUT_NHWC = 0, DP_LAYOUT_NCHW = 1 };
typedef struct dp_preproc_params {
  int32_t batch, in_h, in_w, channels;
  int32_t out_h, out_w;
  int32_t in_dtype, in_layout;
  int32_t out_dtype, out_layout;
  int32_t normalize, reserved;
  float mean[4];
  float stdv[4];
} dp_preproc_params;
int dp_preproc(const dp_preproc_params *p, const void *in, void *out, void *stream);

/* ---- row reductions ------------------------------------------------------
 * rows × cols, reduction over the contiguous last dim (row stride given in
 * elements).  Value kinds write out[rows] (or out[rows, cols] for softmax and
 * the norms).  ARGMAX: first index of the maximum, NaN counts as maximum,
 * output int32 or int64.  RMSNORM: x / sqrt(mean(x²) + eps) · (w + w_offset).
 * LAYERNORM: (x - mean) / sqrt(var + eps) · w + b (biased variance). */
enum {
  DP_RED_SUM = 0, DP_RED_MAX = 1, DP_RED_MIN = 2, DP_RED_MEAN = 3,
  DP_RED_ARGMAX = 4, DP_RED_SOFTMAX = 5, DP_RED_RMSNORM = 6, DP_RED_LAYERNORM = 7
};
typedef struct dp_rowreduce_params {
  int32_t kind, in_dtype, out_dtype, has_weight;
  int32_t has_bias;
  /* softmax / RMSNorm / LayerNorm, fp32 in and out: 1 stores each output row
   * as [hi | hi | lo] (hi = the value with the low 13 mantissa bits cleared,
   * lo = value - hi) at out + row * out_row_stride, blocks cols apart, the
   * operand of a following 3xTF32 product (out_row_stride >= 3 * cols). */
  int32_t out_split;
  int64_t rows, cols;
  int64_t in_row_stride, out_row_stride;
  float eps, weight_offset;
} dp_rowreduce_params;
int dp_rowreduce(const dp_rowreduce_params *p, const void *in, const void *weight,
                 const void *bias, void *out, void *stream);

/* ---- GEMM -----------------------------------------------------------------
 * C[b] = epilogue(A[b] · op(B[b]))  with fp32 accumulation.
 * A: [M, K] row-major (lda).  B: [N, K] row-major when b_layout == DP_B_NK
 * (nn.Linear weight, K contiguous) or [K, N] row-major when DP_B_KN.
 * bf16 × bf16 runs on tcgen05 tensor cores (TMEM accumulator, TMA loads);
 * fp32 × fp32 runs an exact-fp32 FFMA kernel.
 * Epilogue order: × alpha (0 means 1) → + bias[n] → activation →
 * + residual[m, n] (or × residual[m, n] with DP_EPI_MUL: a gated unit whose
 * other half is already computed) → cast to C. */
enum { DP_B_NK = 0, DP_B_KN = 1 };
enum {
  DP_EPI_BIAS = 1, DP_EPI_RELU = 2, DP_EPI_GELU_ERF = 4, DP_EPI_GELU_TANH = 8,
  DP_EPI_RESIDUAL = 16, DP_EPI_SILU = 32,
  /* Row softmax of alpha·(A·Bᵀ) over the N columns (exp via __expf); needs
   * N ≤ 256 (one tensor-core tile holds a whole row), bf16 operands on the
   * tensor-core path and no other epilogue flag. */
  DP_EPI_SOFTMAX = 64,
  /* Multiply by the residual operand instead of adding it (excludes
   * DP_EPI_RESIDUAL). */
  DP_EPI_MUL = 128,
  /* Row argmax of the epilogue's result instead of storing it: each output
   * value (after alpha, bias, activation and residual, rounded to c_dtype)
   * becomes a key (order-preserving bits << 32 | 0xFFFFFFFF - column; NaN
   * ranks highest, -0 ranks with +0) and C is a uint64 key per row, updated
   * with atomicMax, so the largest key is the first column of the maximum.
   * The keys must be zero before the launch and become indices with
   * dp_argmax_keys.  batch 1, tensor-core operands, no softmax.  Fuses the
   * reference's argmax template (templates/reduce.py:11-62) into the GEMM
   * that produces its input: the logits are never written. */
  DP_EPI_ARGMAX = 256,
  /* Store each fp32 result v as the operand of a following 3xTF32 product:
   * C is [M, 3N] (ldc >= 3N) and receives hi = v with the low 13 mantissa
   * bits cleared at columns n and N + n, and lo = v - hi at 2N + n.  fp32 C;
   * dp_gemm_splitk_reduce only (the reduce that finishes a split-K GEMM). */
  DP_EPI_TF32SPLIT = 512
};
typedef struct dp_gemm_params {
  int64_t M, N, K;
  int64_t lda, ldb, ldc, ldr;
  int64_t batch, stride_a, stride_b, stride_c, stride_r;
  int32_t a_dtype, b_dtype, c_dtype, r_dtype;
  int32_t b_layout, epilogue;
  int32_t bias_dtype;
  float alpha;
  /* Two-level batches (e.g. [batch, heads]): when batch2 > 1, matrix z of
   * the batch sits at (z / batch2) * stride_x + (z % batch2) * stride_x2. */
  int64_t batch2, stride_a2, stride_b2, stride_c2, stride_r2;
} dp_gemm_params;
int dp_gemm(const dp_gemm_params *p, const void *A, const void *B, void *C,
            const void *bias, const void *residual, void *stream);

/* ---- split-K reduction ------------------------------------------------------
 * Second half of a GEMM whose K range was split into ``splits`` slices: the
 * first half is dp_gemm batched over the slices (A and B advanced by the
 * slice's K offset, fp32 C = the workspace, no epilogue), which leaves raw
 * partial products in workspace[s][m][n] (slice s at s · slice_stride
 * elements, rows of N).  This sums the slices in slice order (the same bits
 * every run) and applies ``gemm``'s epilogue (alpha, bias, activation,
 * residual or gate operand) and output dtype, writing C [M, N] (ldc).
 * ``gemm.batch`` must be 1.  Same role as the reference's launch_matmul /
 * launch_linear (src/devproc/backend/triton/templates/matmul.py:230-296),
 * which had no split-K. */
typedef struct dp_splitk_params {
  dp_gemm_params gemm;
  int64_t splits, slice_stride;
} dp_splitk_params;
int dp_gemm_splitk_reduce(const dp_splitk_params *p, const void *workspace, void *C, const void *bias,
                          const void *residual, void *stream);

/* ---- stream-K GEMM ------------------------------------------------------
 * dp_gemm for GEMMs whose last wave of output tiles would leave CTA groups
 * idle (e.g. 3,200 x 1,024 with K 4,096: 52 tiles of 256 x 256 for 74 CTA
 * pairs): the K stages of the tiles past the last full wave are dealt out
 * evenly over every group, and the group that computes a tile's last stages
 * adds the earlier groups' fp32 partials (read back in group order, the same
 * bits every run) before the epilogue.  The kernel uses the split only when
 * its cost model picks it for this device and ``workspace_bytes`` holds it;
 * otherwise this is dp_gemm.  The softmax and argmax epilogues never split.
 * ``workspace`` (16-byte aligned, device memory) is scratch for the call:
 * per-tile counters (cleared by the call on ``stream``) and one partial tile
 * per group.  Same role as the reference's launch_matmul / launch_linear
 * (src/devproc/backend/triton/templates/matmul.py:230-296). */
typedef struct dp_streamk_params {
  dp_gemm_params gemm;
  int64_t workspace_bytes;
} dp_streamk_params;
/* Bytes of workspace that always suffice for *p on the current device. */
int dp_gemm_streamk_workspace(const dp_gemm_params *p, int64_t *bytes);
int dp_gemm_streamk(const dp_streamk_params *p, const void *A, const void *B, void *C, const void *bias,
                    const void *residual, void *workspace, void *stream);

/* ---- argmax keys ---------------------------------------------------------
 * mode 0: keys[0..n) = 0 (before a DP_EPI_ARGMAX GEMM); mode 1: out[i] =
 * the column index in keys[i] as out_dtype (DP_I32 or DP_I64). */
typedef struct dp_argmax_keys_params {
  int64_t n;
  int32_t mode, out_dtype;
} dp_argmax_keys_params;
int dp_argmax_keys(const dp_argmax_keys_params *p, void *keys, void *out, void *stream);

/* ---- elementwise region (one kernel per fused IR dataflow region) --------
 * A small register program run per element of an iteration space of up to
 * DP_REGION_MAX_RANK dims.  Operands 0..n_in-1 are inputs, n_in.. are
 * outputs; each has a dtype, per-dim element strides (0 = broadcast) and the
 * element offset of its first element from the bound pointer (a slice of a
 * larger buffer).  Instruction word: opcode | dst << 8 | a << 16 | b << 24. */
#define DP_REGION_MAX_OPERANDS 8
#define DP_REGION_MAX_RANK 6
#define DP_REGION_MAX_INSTR 64
#define DP_REGION_MAX_CONST 32
#define DP_REGION_MAX_REGS 8
enum {
  DP_OP_LOAD = 1,    /* r[dst] = float(operand a)                          */
  DP_OP_STORE = 2,   /* operand a = cast(r[b])                              */
  DP_OP_CONST = 3,   /* r[dst] = consts[a]                                  */
  DP_OP_CHANSEL = 4, /* r[dst] = consts[a + coord[b]]  (per-channel consts) */
  DP_OP_ADD = 10, DP_OP_SUB = 11, DP_OP_MUL = 12, DP_OP_DIV = 13,
  DP_OP_MAX = 14, DP_OP_MIN = 15,
  DP_OP_NEG = 20, DP_OP_ABS = 21, DP_OP_RELU = 22, DP_OP_SIGMOID = 23,
  DP_OP_TANH = 24, DP_OP_EXP = 25, DP_OP_GELU_ERF = 26, DP_OP_GELU_TANH = 27,
  DP_OP_SILU = 28, DP_OP_MOV = 29,
  DP_OP_TF32 = 30    /* keep the 10 mantissa bits a TF32 operand uses (truncate) */
};
typedef struct dp_region_desc {
  int32_t rank, n_in, n_out, n_instr;
  int64_t shape[DP_REGION_MAX_RANK];
  int32_t dtype[DP_REGION_MAX_OPERANDS];
  int64_t stride[DP_REGION_MAX_OPERANDS][DP_REGION_MAX_RANK];
  uint32_t instr[DP_REGION_MAX_INSTR];
  float consts[DP_REGION_MAX_CONST];
  int64_t offset[DP_REGION_MAX_OPERANDS];
} dp_region_desc;
int dp_region(const dp_region_desc *d, const void *const *operands, void *stream);

/* ---- embedding gather -------------------------------------------------------
 * out[i, :] = weight[ids[i], :] for i < n_ids; ids int32 or int64.  An id
 * outside [0, vocab) writes a zero row and sets DP_DEVERR_INDEX. */
typedef struct dp_embedding_params {
  int64_t n_ids, vocab, dim;
  int32_t id_dtype, w_dtype;
} dp_embedding_params;
int dp_embedding(const dp_embedding_params *p, const void *ids, const void *weight,
                 void *out, void *stream);

/* ---- fused attention ----------------------------------------------------------
 * O = softmax(scale · Q·Kᵀ) · V per (batch, key/value head), bf16 in and out,
 * fp32 scores and accumulation, never materialising the scores (one tcgen05
 * kernel: Q·Kᵀ into tensor memory, an online row softmax, P·V accumulated in
 * tensor memory).  Replaces the reference's missing attention (its FX
 * converter had no lowering for scaled_dot_product_attention,
 * src/devproc/ir/fx_converter.py:443-448).
 * Q[b, h, l, :] sits at q + b·q_sb + h·q_sh + l·q_sl (elements), likewise K
 * [b, hk, s], V [b, hk, s] and O [b, h, l].  Query head h uses key/value
 * head h / group; with group > 1 a group's query heads must be stacked rows
 * (q_sh = L·q_sl and o_sh = L·o_sl).  D, Dv ≤ 256, multiples of 8; every
 * row stride and batch / head stride a multiple of 8 elements; bases
 * 16-byte aligned. */
typedef struct dp_attention_params {
  int64_t batch, heads_kv, group;  /* query heads = heads_kv · group */
  int64_t L, S, D, Dv;
  int64_t q_sb, q_sh, q_sl;
  int64_t k_sb, k_sh, k_ss;
  int64_t v_sb, v_sh, v_ss;
  int64_t o_sb, o_sh, o_sl;
  float scale;
  int32_t dtype;  /* DP_BF16 */
} dp_attention_params;
int dp_attention(const dp_attention_params *p, const void *q, const void *k, const void *v, void *o,
                 void *stream);

/* ---- rotary embedding ----------------------------------------------------------
 * Rotate-half rotary position embedding over x viewed as [batch, heads, rows,
 * dim] (element strides; the last dim contiguous), for i < dim/2:
 *   out[.., i]         = x[.., i]·cos[.., i]                 − x[.., i + dim/2]·sin[.., i]
 *   out[.., i + dim/2] = x[.., i + dim/2]·cos[.., i + dim/2] + x[.., i]·sin[.., i + dim/2]
 * each product and sum rounded in fp32, then rounded once to x's type — the
 * torch-level ``devproc::rope`` op.  cos and sin share the strides t_s*
 * (0 broadcasts a dim) and hold dim columns, or dim/2 with half_table (column
 * i serves both halves).  Replaces the slice / neg / cat / mul / add chain the
 * reference's FX converter could not lower (src/devproc/ir/fx_converter.py:
 * 443-448).  x and out: bf16, f16 or f32 (same type); tables bf16, f16 or
 * f32.  dim/2 a multiple of 16 / sizeof(x); strides multiples of that too;
 * bases 16-byte aligned.  out must not overlap x. */
typedef struct dp_rope_params {
  int64_t batch, heads, rows, dim;
  int64_t x_sb, x_sh, x_sr;
  int64_t o_sb, o_sh, o_sr;
  int64_t t_sb, t_sh, t_sr;
  int32_t half_table, x_dtype, t_dtype, reserved;
} dp_rope_params;
int dp_rope(const dp_rope_params *p, const void *x, const void *cos, const void *sin, void *out,
            void *stream);

/* ---- compiled program ------------------------------------------------------
 * A plan is a little-endian blob: dp_plan_header, n_slots × dp_plan_slot,
 * n_records × dp_plan_record.  Slots of kind DP_SLOT_BOUND are caller-owned
 * buffers (inputs, weights, outputs) attached with dp_program_bind; kind
 * DP_SLOT_ARENA slots live at a fixed offset of the program's arena (a
 * multiple of 16 bytes), which dp_program_create allocates once; two arena
 * slots may overlap (a slot can name a column block of another slot's
 * buffer).  dp_program_run enqueues every record in order on the given
 * stream and allocates nothing. */
#define DP_PLAN_MAGIC 0x32425044u /* "DPB2" */
#define DP_PLAN_VERSION 1
#define DP_RECORD_MAX_OPERANDS 8
#define DP_RECORD_PARAM_BYTES 1280
enum { DP_SLOT_BOUND = 0, DP_SLOT_ARENA = 1 };
enum {
  DP_K_PREPROC = 1, DP_K_ROWREDUCE = 2, DP_K_GEMM = 3, DP_K_REGION = 4,
  DP_K_EMBEDDING = 5, DP_K_COPY = 6, DP_K_ATTENTION = 7, DP_K_ROPE = 8, DP_K_SPLITK = 9,
  DP_K_ARGMAX_KEYS = 10, DP_K_GEMM_SK = 11
};
typedef struct dp_plan_header {
  uint32_t magic, version, n_slots, n_records;
  uint64_t arena_bytes, reserved;
} dp_plan_header;
typedef struct dp_plan_slot {
  uint32_t kind, dtype;
  uint64_t offset, bytes;
} dp_plan_slot;
typedef struct dp_plan_record {
  uint32_t kernel, n_operands;
  int32_t operand[DP_RECORD_MAX_OPERANDS];
  uint8_t params[DP_RECORD_PARAM_BYTES];
} dp_plan_record;

typedef struct dp_program dp_program;
int dp_program_create(const void *plan, size_t plan_bytes, int device, dp_program **out);
int dp_program_bind(dp_program *prog, int slot, void *dev_ptr, size_t bytes);
int dp_program_run(dp_program *prog, void *stream);
/* Capture the record sequence into a CUDA graph on first run after binding,
 * then replay it; rebinding any slot drops the graph. */
int dp_program_set_graph(dp_program *prog, int enable);
int dp_program_arena_bytes(const dp_program *prog, uint64_t *bytes);
int dp_program_destroy(dp_program *prog);

/* ---- running a plan without allocating device memory -----------------------
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory at run time — a host application that owns every byte of device
 * memory and hands a plugin only the buffers it reads and writes, or a loop
 * whose owners forbid calls into the driver's allocator: runs ``plan`` once
 * with its intermediate buffers in a fixed array of DP_NOALLOC_ARENA_BYTES in
 * the library's own device memory, present on every GPU that loads the
 * library until the process exits.  ``bound_ptrs`` (and optionally
 * ``bound_bytes``, checked against the slot sizes) give one caller buffer per
 * DP_SLOT_BOUND slot, in slot order: inputs, weights and outputs, and also
 * every sub-range slot of such a buffer (a slice of a weight or an input,
 * listed in the program's meta.json "aliases" as [slot, root slot, byte
 * offset]), which takes the root buffer's pointer plus that offset.  The
 * whole plan and the buffer list are checked before anything is enqueued.  A plan that
 * needs more intermediate bytes than the limit is rejected with
 * DP_ERR_UNSUPPORTED.  No cudaMalloc or cudaFree is called.  The first call on
 * a device (and the first after a cudaDeviceReset) looks up the array's device
 * address, so make it before any stream capture.  Every call shares the one array, which keeps the last call's
 * contents; each intermediate is written before it is read, so nothing needs
 * clearing, but calls that overlap on the GPU (other streams or threads) race
 * on it. */
#define DP_NOALLOC_ARENA_BYTES (64u << 20)
int dp_program_run_noalloc(const void *plan, size_t plan_bytes, void *const *bound_ptrs,
                           const uint64_t *bound_bytes, int n_bound, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* DEVPROC_B200_H */
