// Running a compiled plan without allocating device memory.
//
// dp_program_create allocates the plan's arena (its intermediate buffers)
// with cudaMalloc.  Some callers cannot do that at run time: a host
// application that owns every byte of device memory and hands plugins only
// the buffers they read and write, a latency-critical loop whose owners
// forbid calls into the driver's allocator, or code that must not grow the
// process's device footprint after start-up.  dp_program_run_noalloc runs a
// plan once with its intermediates in g_noalloc_arena, a fixed array in the
// library's own device memory (DP_NOALLOC_ARENA_BYTES on every GPU that loads
// the library, held until the process exits).  The caller still passes every
// input, weight and output buffer.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "dp_common.cuh"

static __device__ __align__(256) uint8_t g_noalloc_arena[DP_NOALLOC_ARENA_BYTES];

namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxSlots = 1024;

struct ArenaAddress {
  unsigned long long ctx_id = 0;  // context the address was looked up in
  void *ptr = nullptr;
};
std::mutex g_noalloc_mu;
ArenaAddress g_noalloc_base[kMaxDevices];

// Device address of g_noalloc_arena on the current device.  In host code the
// symbol itself is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress once per device, with that device current, and cached
// with the id of the context it belongs to: after a cudaDeviceReset the
// device has a new context (and the module a new address), so the lookup is
// made again.  No call here allocates.
int noalloc_base(void **out) {
  int dev = 0;
  DP_CHECK_CUDA(cudaGetDevice(&dev));
  DP_REQUIRE(dev >= 0 && dev < kMaxDevices, DP_ERR_UNSUPPORTED, "dp_program_run_noalloc: device index too large");
  DP_CHECK_CUDA(cudaSetDevice(dev));  // makes the device's primary context current
  // Driver entry points through the runtime, so the library does not link libcuda.
  using GetCurrentFn = CUresult (*)(CUcontext *);
  using GetIdFn = CUresult (*)(CUcontext, unsigned long long *);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  if (!get_current || !get_id) {
    void *a = nullptr, *b = nullptr;
    cudaDriverEntryPointQueryResult qa, qb;
    DP_REQUIRE(cudaGetDriverEntryPoint("cuCtxGetCurrent", &a, cudaEnableDefault, &qa) == cudaSuccess &&
                   qa == cudaDriverEntryPointSuccess &&
                   cudaGetDriverEntryPoint("cuCtxGetId", &b, cudaEnableDefault, &qb) == cudaSuccess &&
                   qb == cudaDriverEntryPointSuccess,
               DP_ERR_CUDA, "dp_program_run_noalloc: cuCtxGetCurrent / cuCtxGetId unavailable");
    get_current = reinterpret_cast<GetCurrentFn>(a);
    get_id = reinterpret_cast<GetIdFn>(b);
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  DP_REQUIRE(get_current(&ctx) == CUDA_SUCCESS && ctx != nullptr && get_id(ctx, &id) == CUDA_SUCCESS,
             DP_ERR_CUDA, "dp_program_run_noalloc: no current CUDA context");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  ArenaAddress &a = g_noalloc_base[dev];
  if (!a.ptr || a.ctx_id != id) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_arena);
    if (e != cudaSuccess) return dp::cuda_status(e, "cudaGetSymbolAddress(g_noalloc_arena)");
    DP_REQUIRE(p != nullptr, DP_ERR_CUDA, "dp_program_run_noalloc: null arena address");
    a.ptr = p;
    a.ctx_id = id;
  }
  *out = a.ptr;
  return DP_OK;
}

int launch_record(const dp_plan_record &rec, const void *const *ops, cudaStream_t s) {
  switch (rec.kernel) {
    case DP_K_PREPROC: {
      dp_preproc_params p;
      memcpy(&p, rec.params, sizeof(p));
      return dp::launch_preproc(p, ops[0], const_cast<void *>(ops[1]), s);
    }
    case DP_K_ROWREDUCE: {
      dp_rowreduce_params p;
      memcpy(&p, rec.params, sizeof(p));
      return dp::launch_rowreduce(p, ops[0], ops[1], ops[2], const_cast<void *>(ops[3]), s);
    }
    case DP_K_GEMM: {
      dp_gemm_params p;
      memcpy(&p, rec.params, sizeof(p));
      return dp::launch_gemm(p, ops[0], ops[1], const_cast<void *>(ops[2]), ops[3], ops[4], s);
    }
    case DP_K_REGION: {
      dp_region_desc d;
      memcpy(&d, rec.params, sizeof(d));
      return dp::launch_region(d, ops, s);
    }
    case DP_K_EMBEDDING: {
      dp_embedding_params p;
      memcpy(&p, rec.params, sizeof(p));
      return dp::launch_embedding(p, ops[0], ops[1], const_cast<void *>(ops[2]), s);
    }
    case DP_K_ATTENTION: {
      dp_attention_params p;
      memcpy(&p, rec.params, sizeof(p));
      return dp::launch_attention(p, ops[0], ops[1], ops[2], const_cast<void *>(ops[3]), s);
    }
    case DP_K_ROPE: {
      dp_rope_params p;
      memcpy(&p, rec.params, sizeof(p));
      return dp::launch_rope(p, ops[0], ops[1], ops[2], const_cast<void *>(ops[3]), s);
    }
    case DP_K_COPY: {
      uint64_t bytes;
      memcpy(&bytes, rec.params, sizeof(bytes));
      cudaError_t e = cudaMemcpyAsync(const_cast<void *>(ops[1]), ops[0], bytes, cudaMemcpyDeviceToDevice, s);
      return e == cudaSuccess ? DP_OK : dp::cuda_status(e, "copy");
    }
    case DP_K_SPLITK: {
      dp_splitk_params p;
      memcpy(&p, rec.params, sizeof(p));
      return dp::launch_splitk_reduce(p, ops[0], const_cast<void *>(ops[1]), ops[2], ops[3], s);
    }
    case DP_K_ARGMAX_KEYS: {
      dp_argmax_keys_params p;
      memcpy(&p, rec.params, sizeof(p));
      return dp::launch_argmax_keys(p, const_cast<void *>(ops[0]), const_cast<void *>(ops[1]), s);
    }
    case DP_K_GEMM_SK: {
      dp_streamk_params p;
      memcpy(&p, rec.params, sizeof(p));
      return dp::launch_gemm_streamk(p, ops[0], ops[1], const_cast<void *>(ops[2]), ops[3], ops[4],
                                     const_cast<void *>(ops[5]), s);
    }
    default:
      return dp::set_error(DP_ERR_PLAN, "unknown record kind " + std::to_string(rec.kernel));
  }
}

}  // namespace

extern "C" int dp_program_run_noalloc(const void *plan, size_t plan_bytes, void *const *bound_ptrs,
                                      const uint64_t *bound_bytes, int n_bound, void *stream) {
  DP_REQUIRE(plan != nullptr, DP_ERR_ARG, "dp_program_run_noalloc: null plan");
  DP_REQUIRE(plan_bytes >= sizeof(dp_plan_header), DP_ERR_PLAN, "plan: truncated header");
  dp_plan_header h;
  memcpy(&h, plan, sizeof(h));
  DP_REQUIRE(h.magic == DP_PLAN_MAGIC, DP_ERR_PLAN, "plan: bad magic");
  DP_REQUIRE(h.version == DP_PLAN_VERSION, DP_ERR_PLAN, "plan: unsupported version");
  DP_REQUIRE(plan_bytes == sizeof(h) + (size_t)h.n_slots * sizeof(dp_plan_slot) +
                               (size_t)h.n_records * sizeof(dp_plan_record),
             DP_ERR_PLAN, "plan: size does not match its header");
  DP_REQUIRE(h.n_slots <= (uint32_t)kMaxSlots, DP_ERR_UNSUPPORTED,
             "dp_program_run_noalloc: plans of more than 1024 slots are not supported");
  DP_REQUIRE(h.arena_bytes <= (uint64_t)DP_NOALLOC_ARENA_BYTES, DP_ERR_UNSUPPORTED,
             "dp_program_run_noalloc: the plan needs " + std::to_string(h.arena_bytes) +
                 " bytes of intermediates; the static arena holds " + std::to_string(DP_NOALLOC_ARENA_BYTES));
  const uint8_t *slots = static_cast<const uint8_t *>(plan) + sizeof(h);
  const uint8_t *records = slots + (size_t)h.n_slots * sizeof(dp_plan_slot);

  // Validate the whole plan and the caller's buffers before anything is
  // enqueued, so a malformed plan writes nothing.
  int n_bound_slots = 0;
  for (uint32_t i = 0; i < h.n_slots; ++i) {
    dp_plan_slot sl;
    memcpy(&sl, slots + i * sizeof(dp_plan_slot), sizeof(sl));
    if (sl.kind == DP_SLOT_ARENA) {
      DP_REQUIRE(sl.offset % 16 == 0 && sl.offset + sl.bytes <= h.arena_bytes, DP_ERR_PLAN,
                 "plan: arena slot " + std::to_string(i) + " out of range or misaligned");
      continue;
    }
    DP_REQUIRE(sl.kind == DP_SLOT_BOUND, DP_ERR_PLAN, "plan: bad kind of slot " + std::to_string(i));
    DP_REQUIRE(bound_ptrs != nullptr && n_bound_slots < n_bound, DP_ERR_ARG,
               "dp_program_run_noalloc: fewer buffers than the plan's bound slots");
    DP_REQUIRE(bound_ptrs[n_bound_slots] != nullptr, DP_ERR_ARG,
               "dp_program_run_noalloc: null buffer " + std::to_string(n_bound_slots));
    DP_REQUIRE(bound_bytes == nullptr || bound_bytes[n_bound_slots] >= sl.bytes, DP_ERR_SHAPE,
               "dp_program_run_noalloc: buffer " + std::to_string(n_bound_slots) + " (slot " + std::to_string(i) +
                   ") is smaller than its slot");
    ++n_bound_slots;
  }
  DP_REQUIRE(n_bound_slots == n_bound, DP_ERR_ARG,
             "dp_program_run_noalloc: " + std::to_string(n_bound) + " buffers for " + std::to_string(n_bound_slots) +
                 " bound slots");
  for (uint32_t r = 0; r < h.n_records; ++r) {
    dp_plan_record rec;
    memcpy(&rec, records + (size_t)r * sizeof(dp_plan_record), sizeof(rec));
    DP_REQUIRE(rec.kernel >= DP_K_PREPROC && rec.kernel <= DP_K_GEMM_SK, DP_ERR_PLAN,
               "program record " + std::to_string(r) + ": unknown record kind " + std::to_string(rec.kernel));
    DP_REQUIRE(rec.n_operands <= DP_RECORD_MAX_OPERANDS, DP_ERR_PLAN,
               "program record " + std::to_string(r) + ": too many operands");
    for (uint32_t i = 0; i < rec.n_operands; ++i)
      DP_REQUIRE(rec.operand[i] >= -1 && rec.operand[i] < (int32_t)h.n_slots, DP_ERR_PLAN,
                 "program record " + std::to_string(r) + ": operand out of range");
  }

  void *base = nullptr;
  int st = noalloc_base(&base);
  if (st != DP_OK) return st;

  // Resolve every slot: caller buffers in slot order, intermediates in the arena.
  void *ptr[kMaxSlots];
  int next_bound = 0;
  for (uint32_t i = 0; i < h.n_slots; ++i) {
    dp_plan_slot sl;
    memcpy(&sl, slots + i * sizeof(dp_plan_slot), sizeof(sl));
    ptr[i] = sl.kind == DP_SLOT_ARENA ? static_cast<uint8_t *>(base) + sl.offset : bound_ptrs[next_bound++];
  }

  cudaStream_t s = dp::as_stream(stream);
  for (uint32_t r = 0; r < h.n_records; ++r) {
    dp_plan_record rec;
    memcpy(&rec, records + (size_t)r * sizeof(dp_plan_record), sizeof(rec));
    const void *ops[DP_RECORD_MAX_OPERANDS] = {nullptr};
    for (uint32_t i = 0; i < rec.n_operands; ++i) ops[i] = rec.operand[i] >= 0 ? ptr[rec.operand[i]] : nullptr;
    st = launch_record(rec, ops, s);
    if (st != DP_OK) {
      char buf[512];
      dp_last_error(buf, sizeof(buf));
      return dp::set_error(st, "program record " + std::to_string(r) + ": " + buf);
    }
  }
  return DP_OK;
}
