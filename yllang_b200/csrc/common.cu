// Host-side plumbing shared by the store and index entry points.
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace ylk {

namespace {
thread_local std::string g_last_error;
std::mutex g_sm_mutex;
std::vector<int> g_sm_count;  // per device ordinal, 0 = not queried yet
}  // namespace

void set_last_error(const std::string &msg) { g_last_error = msg; }
void clear_last_error() { g_last_error.clear(); }

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return dev;
}

int sm_count() {
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_sm_mutex);
  if (static_cast<int>(g_sm_count.size()) <= dev) g_sm_count.resize(dev + 1, 0);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;  // B200
    }
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

uint64_t bulk_wait_limit_ns() {
  static const uint64_t limit = [] {
    const char *e = std::getenv("YL_BULK_WAIT_LIMIT_NS");
    if (e == nullptr || *e == '\0') return kBulkWaitLimitNs;
    char *end = nullptr;
    const unsigned long long v = std::strtoull(e, &end, 10);
    return (end != e && *end == '\0' && v > 0 && v <= kBulkWaitLimitNs) ? static_cast<uint64_t>(v) : kBulkWaitLimitNs;
  }();
  return limit;
}

}  // namespace ylk

extern "C" {

const char *yl_status_string(int status) {
  switch (status) {
    case YL_OK: return "YL_OK";
    case YL_ERR_NULL_ARG: return "YL_ERR_NULL_ARG";
    case YL_ERR_BAD_SIZE: return "YL_ERR_BAD_SIZE";
    case YL_ERR_ALIGNMENT: return "YL_ERR_ALIGNMENT";
    case YL_ERR_UNSUPPORTED: return "YL_ERR_UNSUPPORTED";
    case YL_ERR_CUDA: return "YL_ERR_CUDA";
    default: return "YL_ERR_UNKNOWN";
  }
}

const char *yl_last_error(void) { return ylk::g_last_error.c_str(); }

int yl_abi_version(void) { return YL_KVPATH_ABI_VERSION; }

}  // extern "C"
