// Library-level C ABI: version, per-thread last error, device set-up and the
// device error word.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "dp_common.cuh"

__device__ unsigned int g_dp_err_code = 0;
__device__ long long g_dp_err_info = 0;

namespace dp {

namespace {
thread_local std::string t_last_error;
}

int set_error(int code, const std::string &msg) {
  t_last_error = msg;
  return code;
}

int cuda_status(cudaError_t e, const char *what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return set_error(DP_ERR_CUDA, m);
}

int num_sms() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace dp

extern "C" int dp_version(void) { return DP_ABI_VERSION * 10000 + 1; }

extern "C" int dp_last_error(char *buf, size_t buf_len) {
  if (!buf || buf_len == 0) return DP_ERR_ARG;
  const std::string &m = dp::t_last_error;
  size_t n = m.size() < buf_len - 1 ? m.size() : buf_len - 1;
  memcpy(buf, m.data(), n);
  buf[n] = '\0';
  return DP_OK;
}

extern "C" int dp_device_init(int device) {
  int count = 0;
  DP_CHECK_CUDA(cudaGetDeviceCount(&count));
  DP_REQUIRE(device >= 0 && device < count, DP_ERR_ARG,
             "dp_device_init: device " + std::to_string(device) + " not present (" + std::to_string(count) +
                 " visible)");
  DP_CHECK_CUDA(cudaSetDevice(device));
  int major = 0, minor = 0;
  DP_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  DP_CHECK_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  DP_REQUIRE(major == 10 && minor == 0, DP_ERR_UNSUPPORTED,
             "dp_device_init: this library is built for sm_100a (B200); device is sm_" + std::to_string(major) +
                 std::to_string(minor));
  return DP_OK;
}

extern "C" int dp_device_error(int *code, int64_t *info) {
  DP_REQUIRE(code != nullptr, DP_ERR_ARG, "dp_device_error: null code");
  DP_CHECK_CUDA(cudaDeviceSynchronize());
  unsigned int c = 0;
  long long i = 0;
  DP_CHECK_CUDA(cudaMemcpyFromSymbol(&c, g_dp_err_code, sizeof(c)));
  DP_CHECK_CUDA(cudaMemcpyFromSymbol(&i, g_dp_err_info, sizeof(i)));
  const unsigned int zero = 0;
  const long long zero64 = 0;
  DP_CHECK_CUDA(cudaMemcpyToSymbol(g_dp_err_code, &zero, sizeof(zero)));
  DP_CHECK_CUDA(cudaMemcpyToSymbol(g_dp_err_info, &zero64, sizeof(zero64)));
  *code = (int)c;
  if (info) *info = (int64_t)i;
  return DP_OK;
}
