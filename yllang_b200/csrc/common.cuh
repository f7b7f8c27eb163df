// Shared host/device helpers of the C-ABI library: status plumbing, per-device
// launch facts, and a multiply-shift divider for row -> (plane, token) splits.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "yl_kvpath.h"

namespace ylk {

// ---------------------------------------------------------------------------
// Host-side status: every entry point returns a yl_status and leaves a detail
// string that yl_last_error() hands back (per host thread).
// ---------------------------------------------------------------------------
void set_last_error(const std::string &msg);
void clear_last_error();

inline int fail(int status, const char *fmt, long long a = 0, long long b = 0) {
  char buf[256];
  std::snprintf(buf, sizeof(buf), fmt, a, b);
  set_last_error(buf);
  return status;
}

inline int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(std::string(what) + ": " + cudaGetErrorString(e));
    return YL_ERR_CUDA;
  }
  return YL_OK;
}

// Number of SMs of the current device (cached per device ordinal).
int sm_count();

// Bound of a bulk-copy kernel's wait for its own copies (mbarrier phase):
// 2 s of %globaltimer, after which the waiting thread sets YL_DEVERR_TIMEOUT,
// waits once more with the full bound so its copies land, and leaves.
// YL_BULK_WAIT_LIMIT_NS (read once per process; 1 .. 2e9) lowers the first of
// those waits in the store's and the step's bulk-copy kernels, so a test can
// make it give up while the copies are still in flight.
constexpr uint64_t kBulkWaitLimitNs = 2000000000ull;
uint64_t bulk_wait_limit_ns();
// Current device ordinal (cached per host thread would be wrong across
// cudaSetDevice, so this is a plain query).
int current_device();

// ---------------------------------------------------------------------------
// Division by a run-time invariant divisor d >= 1 for dividends n < 2^31:
//   q = (umulhi(m, n) + n) >> s,   s = ceil(log2 d),
//   m = floor(2^32 * (2^s - d) / d) + 1          (taken mod 2^32)
// This is the round-up multiplier of Granlund & Montgomery, "Division by
// Invariant Integers using Multiplication" (PLDI 1994), Fig. 4.1; the sum
// umulhi(m, n) + n cannot wrap because umulhi(m, n) < n < 2^31.
// ---------------------------------------------------------------------------
struct FastDiv {
  uint32_t d;
  uint32_t m;
  uint32_t s;

  FastDiv() = default;
  __host__ explicit FastDiv(uint32_t divisor) : d(divisor), m(0), s(0) {
    while ((1ull << s) < divisor) ++s;
    const uint64_t two_s = 1ull << s;
    m = static_cast<uint32_t>(((two_s - divisor) << 32) / divisor + 1);
  }
  __host__ __device__ __forceinline__ uint32_t div(uint32_t n) const {
#ifdef __CUDA_ARCH__
    return (__umulhi(m, n) + n) >> s;
#else
    return static_cast<uint32_t>(((static_cast<uint64_t>(m) * n >> 32) + n) >> s);
#endif
  }
};

// Programmatic dependent launch.  A kernel launched with the
// programmatic-stream-serialization attribute may start while the kernel
// before it in the stream is still running: pdl_wait() blocks the calling
// thread until that kernel has completed and its writes are visible (it
// returns at once for a normal launch), and pdl_trigger() lets the next such
// kernel start launching early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Launch `kernel` as a programmatic dependent of the kernel before it on the
// stream: its blocks may be placed while that kernel drains, which hides the
// launch.  The kernel must call pdl_wait() before it touches memory an
// earlier kernel may have written (for a normal launch the wait returns at
// once), so stream order is kept.  Returns a yl_status.
template <typename... KArgs, typename... Args>
inline int launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                            const char *what, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_last_error(std::string(what) + ": " + cudaGetErrorString(e));
    return YL_ERR_CUDA;
  }
  return check_launch(what);
}

__device__ __forceinline__ void raise_deverr(uint32_t *word, uint32_t bit) {
  if (word != nullptr) atomicOr(word, bit);
}

}  // namespace ylk
