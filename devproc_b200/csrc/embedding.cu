// Embedding gather: out[i, :] = weight[ids[i], :].
//
// No reference kernel exists: the reference's FX converter rejected
// ``embedding`` (src/devproc/ir/fx_converter.py:197-199).  One warp copies one
// row with 16-byte vector moves when the row size and pointers allow it.  An
// id outside [0, vocab) writes a zero row and records DP_DEVERR_INDEX with
// the position of the first bad id (torch raises IndexError there).
#include "dp_common.cuh"

namespace dpk_embedding {

template <typename V>
__global__ void __launch_bounds__(256) gather_kernel(dp_embedding_params p, const void *__restrict__ ids,
                                                     const V *__restrict__ w, V *__restrict__ out,
                                                     int64_t row_vecs) {
  dp::pdl_trigger();
  dp::pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t i = warp; i < p.n_ids; i += nwarps) {
    const long long id = p.id_dtype == DP_I64 ? reinterpret_cast<const long long *>(ids)[i]
                                              : (long long)reinterpret_cast<const int32_t *>(ids)[i];
    V *dst = out + i * row_vecs;
    if (id < 0 || id >= p.vocab) {
      if (lane == 0) dp_report(DP_DEVERR_INDEX, i);
      for (int64_t c = lane; c < row_vecs; c += 32) dst[c] = V{};
      continue;
    }
    const V *src = w + id * row_vecs;
    for (int64_t c = lane; c < row_vecs; c += 32) dst[c] = __ldg(src + c);
  }
}

}  // namespace dpk_embedding

namespace dp {

int launch_embedding(const dp_embedding_params &p, const void *ids, const void *w, void *out, cudaStream_t s) {
  using namespace dpk_embedding;
  DP_REQUIRE(ids && w && out, DP_ERR_ARG, "embedding: null pointer");
  DP_REQUIRE(p.n_ids > 0 && p.vocab > 0 && p.dim > 0, DP_ERR_SHAPE, "embedding: sizes must be positive");
  DP_REQUIRE(p.id_dtype == DP_I32 || p.id_dtype == DP_I64, DP_ERR_ARG, "embedding: ids must be int32/int64");
  const int eb = dtype_bytes(p.w_dtype);
  DP_REQUIRE(eb > 0, DP_ERR_ARG, "embedding: bad weight dtype");
  const int64_t row_bytes = p.dim * eb;
  int64_t warps = p.n_ids;
  int64_t blocks = (warps * 32 + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  auto aligned = [](const void *q, int a) { return reinterpret_cast<uintptr_t>(q) % a == 0; };
  if (row_bytes % 16 == 0 && aligned(w, 16) && aligned(out, 16)) {
    dp::launch_k(gather_kernel<uint4>, (int)blocks, 256, 0, s, p, ids, static_cast<const uint4 *>(w),
                                                    static_cast<uint4 *>(out), row_bytes / 16);
  } else if (row_bytes % 4 == 0 && aligned(w, 4) && aligned(out, 4)) {
    dp::launch_k(gather_kernel<uint32_t>, (int)blocks, 256, 0, s, p, ids, static_cast<const uint32_t *>(w),
                                                       static_cast<uint32_t *>(out), row_bytes / 4);
  } else {
    dp::launch_k(gather_kernel<uint8_t>, (int)blocks, 256, 0, s, p, ids, static_cast<const uint8_t *>(w),
                                                      static_cast<uint8_t *>(out), row_bytes);
  }
  DP_CHECK_CUDA(cudaGetLastError());
  return DP_OK;
}

}  // namespace dp

extern "C" int dp_embedding(const dp_embedding_params *p, const void *ids, const void *weight, void *out,
                            void *stream) {
  if (!p) return dp::set_error(DP_ERR_ARG, "dp_embedding: null params");
  return dp::launch_embedding(*p, ids, weight, out, dp::as_stream(stream));
}
