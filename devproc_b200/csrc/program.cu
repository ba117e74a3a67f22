// Compiled-program executor: a plan of launch records over a static arena.
//
// Replaces TritonCompiledProgram.run / _run_jit_with_ir
// (src/devproc/backend/triton/compiler.py:54-68, 206-250), which allocated
// every value with torch.empty on every call (memory.py:35) and re-launched
// all earlier kernels after each op (compiler.py:352-355), and the ctypes
// launcher that was never reached (runtime/kernel_launcher.py:59-273).
//
// dp_program_create parses and validates the whole plan once and allocates
// the arena once; dp_program_run only resolves pointers and enqueues the
// records on the caller's stream (or replays them as one CUDA graph).
#include <cstring>
#include <vector>

#include "dp_common.cuh"

struct dp_program {
  int device = 0;
  uint64_t arena_bytes = 0;
  void *arena = nullptr;
  std::vector<dp_plan_slot> slots;
  std::vector<dp_plan_record> records;
  std::vector<void *> ptr;
  std::vector<uint8_t> bound;
  bool use_graph = false;
  int eager_runs = 0;  // runs since the last (re)bind
  cudaGraphExec_t exec = nullptr;
  cudaStream_t exec_stream = nullptr;

  void drop_graph() {
    if (exec) cudaGraphExecDestroy(exec);
    exec = nullptr;
    exec_stream = nullptr;
    eager_runs = 0;
  }
};

namespace {

int run_records(dp_program *prog, cudaStream_t s) {
  for (size_t r = 0; r < prog->records.size(); ++r) {
    const dp_plan_record &rec = prog->records[r];
    const void *ops[DP_RECORD_MAX_OPERANDS] = {nullptr};
    for (uint32_t i = 0; i < rec.n_operands; ++i)
      ops[i] = rec.operand[i] >= 0 ? prog->ptr[rec.operand[i]] : nullptr;
    int st = DP_OK;
    switch (rec.kernel) {
      case DP_K_PREPROC: {
        dp_preproc_params p;
        memcpy(&p, rec.params, sizeof(p));
        st = dp::launch_preproc(p, ops[0], const_cast<void *>(ops[1]), s);
        break;
      }
      case DP_K_ROWREDUCE: {
        dp_rowreduce_params p;
        memcpy(&p, rec.params, sizeof(p));
        st = dp::launch_rowreduce(p, ops[0], ops[1], ops[2], const_cast<void *>(ops[3]), s);
        break;
      }
      case DP_K_GEMM: {
        dp_gemm_params p;
        memcpy(&p, rec.params, sizeof(p));
        st = dp::launch_gemm(p, ops[0], ops[1], const_cast<void *>(ops[2]), ops[3], ops[4], s);
        break;
      }
      case DP_K_REGION: {
        dp_region_desc d;
        memcpy(&d, rec.params, sizeof(d));
        st = dp::launch_region(d, ops, s);
        break;
      }
      case DP_K_EMBEDDING: {
        dp_embedding_params p;
        memcpy(&p, rec.params, sizeof(p));
        st = dp::launch_embedding(p, ops[0], ops[1], const_cast<void *>(ops[2]), s);
        break;
      }
      case DP_K_ATTENTION: {
        dp_attention_params p;
        memcpy(&p, rec.params, sizeof(p));
        st = dp::launch_attention(p, ops[0], ops[1], ops[2], const_cast<void *>(ops[3]), s);
        break;
      }
      case DP_K_ROPE: {
        dp_rope_params p;
        memcpy(&p, rec.params, sizeof(p));
        st = dp::launch_rope(p, ops[0], ops[1], ops[2], const_cast<void *>(ops[3]), s);
        break;
      }
      case DP_K_COPY: {
        uint64_t bytes;
        memcpy(&bytes, rec.params, sizeof(bytes));
        cudaError_t e = cudaMemcpyAsync(const_cast<void *>(ops[1]), ops[0], bytes, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) st = dp::cuda_status(e, "program copy record");
        break;
      }
      case DP_K_SPLITK: {
        dp_splitk_params p;
        memcpy(&p, rec.params, sizeof(p));
        st = dp::launch_splitk_reduce(p, ops[0], const_cast<void *>(ops[1]), ops[2], ops[3], s);
        break;
      }
      case DP_K_ARGMAX_KEYS: {
        dp_argmax_keys_params p;
        memcpy(&p, rec.params, sizeof(p));
        st = dp::launch_argmax_keys(p, const_cast<void *>(ops[0]), const_cast<void *>(ops[1]), s);
        break;
      }
      case DP_K_GEMM_SK: {
        dp_streamk_params p;
        memcpy(&p, rec.params, sizeof(p));
        st = dp::launch_gemm_streamk(p, ops[0], ops[1], const_cast<void *>(ops[2]), ops[3], ops[4],
                                     const_cast<void *>(ops[5]), s);
        break;
      }
      default:
        st = dp::set_error(DP_ERR_PLAN, "program: unknown record kind " + std::to_string(rec.kernel));
    }
    if (st != DP_OK) {
      char buf[512];
      dp_last_error(buf, sizeof(buf));
      return dp::set_error(st, "program record " + std::to_string(r) + ": " + buf);
    }
  }
  return DP_OK;
}

}  // namespace

extern "C" int dp_program_create(const void *plan, size_t plan_bytes, int device, dp_program **out) {
  DP_REQUIRE(plan && out, DP_ERR_ARG, "dp_program_create: null argument");
  *out = nullptr;
  DP_REQUIRE(plan_bytes >= sizeof(dp_plan_header), DP_ERR_PLAN, "plan: truncated header");
  dp_plan_header h;
  memcpy(&h, plan, sizeof(h));
  DP_REQUIRE(h.magic == DP_PLAN_MAGIC, DP_ERR_PLAN, "plan: bad magic");
  DP_REQUIRE(h.version == DP_PLAN_VERSION, DP_ERR_PLAN, "plan: unsupported version " + std::to_string(h.version));
  const size_t need = sizeof(h) + (size_t)h.n_slots * sizeof(dp_plan_slot) +
                      (size_t)h.n_records * sizeof(dp_plan_record);
  DP_REQUIRE(plan_bytes == need, DP_ERR_PLAN,
             "plan: size " + std::to_string(plan_bytes) + " != expected " + std::to_string(need));
  auto prog = new dp_program();
  prog->device = device;
  prog->arena_bytes = h.arena_bytes;
  const uint8_t *cur = static_cast<const uint8_t *>(plan) + sizeof(h);
  prog->slots.resize(h.n_slots);
  if (h.n_slots) memcpy(prog->slots.data(), cur, h.n_slots * sizeof(dp_plan_slot));
  cur += h.n_slots * sizeof(dp_plan_slot);
  prog->records.resize(h.n_records);
  if (h.n_records) memcpy(prog->records.data(), cur, h.n_records * sizeof(dp_plan_record));
  auto fail = [&](int code, const std::string &m) {
    delete prog;
    return dp::set_error(code, m);
  };
  for (uint32_t i = 0; i < h.n_slots; ++i) {
    const dp_plan_slot &sl = prog->slots[i];
    if (sl.kind != DP_SLOT_BOUND && sl.kind != DP_SLOT_ARENA) return fail(DP_ERR_PLAN, "plan: bad slot kind");
    if (sl.kind == DP_SLOT_ARENA && (sl.offset % 16 != 0 || sl.offset + sl.bytes > h.arena_bytes))
      return fail(DP_ERR_PLAN, "plan: arena slot " + std::to_string(i) + " out of range or misaligned");
  }
  for (uint32_t r = 0; r < h.n_records; ++r) {
    const dp_plan_record &rec = prog->records[r];
    if (rec.n_operands > DP_RECORD_MAX_OPERANDS) return fail(DP_ERR_PLAN, "plan: too many operands");
    for (uint32_t i = 0; i < rec.n_operands; ++i)
      if (rec.operand[i] < -1 || rec.operand[i] >= (int32_t)h.n_slots)
        return fail(DP_ERR_PLAN, "plan: record " + std::to_string(r) + " operand out of range");
  }
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    delete prog;
    return dp::cuda_status(e, "cudaSetDevice");
  }
  if (h.arena_bytes) {
    e = cudaMalloc(&prog->arena, h.arena_bytes);
    if (e != cudaSuccess) {
      delete prog;
      return dp::cuda_status(e, "arena cudaMalloc");
    }
  }
  prog->ptr.assign(h.n_slots, nullptr);
  prog->bound.assign(h.n_slots, 0);
  for (uint32_t i = 0; i < h.n_slots; ++i)
    if (prog->slots[i].kind == DP_SLOT_ARENA) {
      prog->ptr[i] = static_cast<uint8_t *>(prog->arena) + prog->slots[i].offset;
      prog->bound[i] = 1;
    }
  *out = prog;
  return DP_OK;
}

extern "C" int dp_program_bind(dp_program *prog, int slot, void *dev_ptr, size_t bytes) {
  DP_REQUIRE(prog, DP_ERR_ARG, "dp_program_bind: null program");
  DP_REQUIRE(slot >= 0 && slot < (int)prog->slots.size(), DP_ERR_ARG, "dp_program_bind: slot out of range");
  DP_REQUIRE(prog->slots[slot].kind == DP_SLOT_BOUND, DP_ERR_ARG, "dp_program_bind: slot is an arena slot");
  DP_REQUIRE(dev_ptr != nullptr, DP_ERR_ARG, "dp_program_bind: null pointer");
  DP_REQUIRE(bytes >= prog->slots[slot].bytes, DP_ERR_SHAPE,
             "dp_program_bind: slot " + std::to_string(slot) + " needs " + std::to_string(prog->slots[slot].bytes) +
                 " bytes, got " + std::to_string(bytes));
  if (prog->ptr[slot] != dev_ptr) prog->drop_graph();
  prog->ptr[slot] = dev_ptr;
  prog->bound[slot] = 1;
  return DP_OK;
}

extern "C" int dp_program_set_graph(dp_program *prog, int enable) {
  DP_REQUIRE(prog, DP_ERR_ARG, "dp_program_set_graph: null program");
  prog->use_graph = enable != 0;
  prog->drop_graph();
  return DP_OK;
}

extern "C" int dp_program_run(dp_program *prog, void *stream) {
  DP_REQUIRE(prog, DP_ERR_ARG, "dp_program_run: null program");
  for (size_t i = 0; i < prog->bound.size(); ++i)
    DP_REQUIRE(prog->bound[i], DP_ERR_STATE, "dp_program_run: slot " + std::to_string(i) + " is not bound");
  cudaStream_t s = dp::as_stream(stream);
  DP_CHECK_CUDA(cudaSetDevice(prog->device));
  if (!prog->use_graph || s == nullptr) return run_records(prog, s);
  if (prog->exec && prog->exec_stream == s) {
    DP_CHECK_CUDA(cudaGraphLaunch(prog->exec, s));
    return DP_OK;
  }
  if (prog->eager_runs == 0) {  // first run after (re)binding: eager, loads every kernel
    int st = run_records(prog, s);
    if (st == DP_OK) prog->eager_runs = 1;
    return st;
  }
  prog->drop_graph();
  DP_CHECK_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int st = run_records(prog, s);
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(s, &graph);
  if (st != DP_OK) {
    if (graph) cudaGraphDestroy(graph);
    return st;
  }
  if (e != cudaSuccess) return dp::cuda_status(e, "cudaStreamEndCapture");
  e = cudaGraphInstantiate(&prog->exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    prog->exec = nullptr;
    return dp::cuda_status(e, "cudaGraphInstantiate");
  }
  prog->exec_stream = s;
  prog->eager_runs = 1;
  DP_CHECK_CUDA(cudaGraphLaunch(prog->exec, s));
  return DP_OK;
}

extern "C" int dp_program_arena_bytes(const dp_program *prog, uint64_t *bytes) {
  DP_REQUIRE(prog && bytes, DP_ERR_ARG, "dp_program_arena_bytes: null argument");
  *bytes = prog->arena_bytes;
  return DP_OK;
}

extern "C" int dp_program_destroy(dp_program *prog) {
  if (!prog) return DP_OK;
  prog->drop_graph();
  int st = DP_OK;
  if (prog->arena) {
    cudaSetDevice(prog->device);
    cudaError_t e = cudaFree(prog->arena);
    if (e != cudaSuccess) st = dp::cuda_status(e, "arena cudaFree");
  }
  delete prog;
  return st;
}
