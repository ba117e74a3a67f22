// Library-level C ABI: version, per-thread last error, device set-up and the
// device error word.
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "dp_common.cuh"

__device__ unsigned int g_dp_err_code = 0;
__device__ long long g_dp_err_info = 0;
__device__ int *g_dp_err_host = nullptr;
__device__ unsigned long long g_dp_wait_limit_ns = 2000000000ull;
__device__ unsigned int g_dp_withhold_copies = 0;

namespace {
constexpr int kMaxDevices = 64;
constexpr unsigned long long kDefaultWaitLimitNs = 2000000000ull;
std::mutex g_host_word_mu;
int *g_host_word[kMaxDevices] = {nullptr};  // pinned, mapped; one per initialised device

int current_device(int *dev) {
  DP_CHECK_CUDA(cudaGetDevice(dev));
  DP_REQUIRE(*dev >= 0 && *dev < kMaxDevices, DP_ERR_UNSUPPORTED, "device ordinal above 63");
  return DP_OK;
}
}  // namespace

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

int kernel_blocks_per_sm(const void *func, int threads, size_t smem, bool max_carveout, int *per_sm) {
  struct Key {
    int dev, threads;
    const void *func;
    size_t smem;
    bool operator<(const Key &o) const {
      if (dev != o.dev) return dev < o.dev;
      if (func != o.func) return func < o.func;
      if (threads != o.threads) return threads < o.threads;
      return smem < o.smem;
    }
  };
  static std::mutex mu;
  static std::map<Key, int> cache;
  int dev = 0;
  DP_CHECK_CUDA(cudaGetDevice(&dev));
  const Key k{dev, threads, func, smem};
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(k);
  if (it != cache.end()) {
    *per_sm = it->second;
    return DP_OK;
  }
  // The opt-in only ever grows, so a smaller launch never revokes a larger
  // one's.  It is granted for every size: static shared memory (barriers)
  // counts against the same 48 KB default as the dynamic bytes.
  static std::map<std::pair<int, const void *>, size_t> granted;
  size_t &g = granted[{dev, func}];
  if (smem > g) {
    DP_CHECK_CUDA(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    g = smem;
  }
  if (max_carveout)
    DP_CHECK_CUDA(cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       (int)cudaSharedmemCarveoutMaxShared));
  int n = 0;
  DP_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, func, threads, smem));
  if (n < 1) n = 1;
  cache.emplace(k, n);
  *per_sm = n;
  return DP_OK;
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
  DP_REQUIRE(device < kMaxDevices, DP_ERR_UNSUPPORTED, "dp_device_init: device ordinal above 63");
  // The host mirror of the error word: allocated once per device, its device
  // address (re)written into this device's g_dp_err_host on every init.
  std::lock_guard<std::mutex> lk(g_host_word_mu);
  if (!g_host_word[device]) {
    int *h = nullptr;
    DP_CHECK_CUDA(cudaHostAlloc(reinterpret_cast<void **>(&h), sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable));
    *reinterpret_cast<volatile int *>(h) = 0;
    g_host_word[device] = h;
  }
  int *d = nullptr;
  DP_CHECK_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void **>(&d), g_host_word[device], 0));
  DP_CHECK_CUDA(cudaMemcpyToSymbol(g_dp_err_host, &d, sizeof(d)));
  return DP_OK;
}

extern "C" int dp_device_error_pending(int device, int *code) {
  DP_REQUIRE(code != nullptr, DP_ERR_ARG, "dp_device_error_pending: null code");
  DP_REQUIRE(device >= 0 && device < kMaxDevices, DP_ERR_ARG, "dp_device_error_pending: bad device");
  const int *h = g_host_word[device];
  *code = h ? *reinterpret_cast<const volatile int *>(h) : 0;
  return DP_OK;
}

extern "C" int dp_set_wait_limit(int device, uint64_t limit_ns) {
  DP_REQUIRE(device >= 0 && device < kMaxDevices, DP_ERR_ARG, "dp_set_wait_limit: bad device");
  DP_CHECK_CUDA(cudaSetDevice(device));
  const unsigned long long v = limit_ns ? (unsigned long long)limit_ns : kDefaultWaitLimitNs;
  DP_CHECK_CUDA(cudaMemcpyToSymbol(g_dp_wait_limit_ns, &v, sizeof(v)));
  return DP_OK;
}

extern "C" int dp_test_withhold_copies(int device, int enable) {
  DP_REQUIRE(device >= 0 && device < kMaxDevices, DP_ERR_ARG, "dp_test_withhold_copies: bad device");
  DP_CHECK_CUDA(cudaSetDevice(device));
  const unsigned int v = enable ? 1u : 0u;
  DP_CHECK_CUDA(cudaMemcpyToSymbol(g_dp_withhold_copies, &v, sizeof(v)));
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
  int dev = 0;
  int st = current_device(&dev);
  if (st != DP_OK) return st;
  if (g_host_word[dev]) *reinterpret_cast<volatile int *>(g_host_word[dev]) = 0;
  *code = (int)c;
  if (info) *info = (int64_t)i;
  return DP_OK;
}
