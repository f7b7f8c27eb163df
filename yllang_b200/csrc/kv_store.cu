// Paged KV-cache store for sm_100a: scatter each step's new K/V rows into the
// layer-major pool by slot mapping.
//
// Reference behaviour (src/kvcache/store_kv_cache.cu:46-77): for i < N,
// k_cache[idx[i]] <- k[i] and v_cache[idx[i]] <- v[i], one warp per token with
// 16-byte vector copies, one launch per layer.  Here one launch can cover all
// layers of a step, every thread keeps several independent row loads in
// flight before its stores (the copy is HBM-latency bound, so bytes in flight
// per SM set the achieved bandwidth), and small rows are split over sub-warp
// lane groups so no lane idles.
//
// Work decomposition: the rows to copy are enumerated plane-major,
//     row r in [0, 2 * L * N):  plane = r / N (plane = 2 * layer + {0: K, 1: V}),
//                               token = r % N,
// so neighbouring lane groups copy neighbouring tokens of one plane (for a
// prefill chunk their destinations are neighbouring slots of one page).  A
// group of G lanes copies one row as G * VPL vectors of W bytes; a group takes
// R rows per iteration, issuing all R * VPL loads before any store.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace ylk {

struct StoreParams {
  const char *k;
  const char *v;
  char *k_cache;
  char *v_cache;
  const void *slots;
  int64_t k_row_stride;
  int64_t v_row_stride;
  int64_t cache_row_stride;
  int64_t k_layer_stride;
  int64_t v_layer_stride;
  int64_t cache_layer_stride;
  int64_t num_slots;
  uint32_t *error_word;
  uint32_t total_rows;  // 2 * L * N  (< 2^31)
  uint32_t row_units;   // row_bytes / unit, generic kernel only
  FastDiv by_tokens;    // divides a row id by N
};

// ---------------------------------------------------------------------------
// Vector types and cache-hinted global accesses.  Loads of the step's input
// rows are read exactly once: non-coherent path, no L1 allocation.
// ---------------------------------------------------------------------------
template <int W>
struct Vec;
template <>
struct Vec<16> {
  uint32_t r[4];
};
template <>
struct Vec<32> {
  uint32_t r[8];
};

__device__ __forceinline__ void load_vec(Vec<16> &x, const char *p) {
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(x.r[0]), "=r"(x.r[1]), "=r"(x.r[2]), "=r"(x.r[3])
               : "l"(p));
}
__device__ __forceinline__ void store_vec(char *p, const Vec<16> &x) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(x.r[0]), "r"(x.r[1]), "r"(x.r[2]),
               "r"(x.r[3])
               : "memory");
}
__device__ __forceinline__ void load_vec(Vec<32> &x, const char *p) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(x.r[0]), "=r"(x.r[1]), "=r"(x.r[2]), "=r"(x.r[3]), "=r"(x.r[4]), "=r"(x.r[5]),
                 "=r"(x.r[6]), "=r"(x.r[7])
               : "l"(p));
}
__device__ __forceinline__ void store_vec(char *p, const Vec<32> &x) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(x.r[0]), "r"(x.r[1]),
               "r"(x.r[2]), "r"(x.r[3]), "r"(x.r[4]), "r"(x.r[5]), "r"(x.r[6]), "r"(x.r[7])
               : "memory");
}

template <typename SlotT>
__device__ __forceinline__ int64_t load_slot(const void *slots, uint32_t token) {
  return static_cast<int64_t>(__ldg(static_cast<const SlotT *>(slots) + token));
}

// True when the slot names a pool row; -1 (padding) is skipped silently and
// anything else out of range is skipped and reported.
__device__ __forceinline__ bool slot_ok(int64_t slot, const StoreParams &p) {
  if (slot >= 0 && (p.num_slots <= 0 || slot < p.num_slots)) return true;
  if (slot != -1) raise_deverr(p.error_word, YL_DEVERR_SLOT_RANGE);
  return false;
}

struct RowAddr {
  const char *src;
  char *dst_base;  // pool base of this plane's layer; slot offset added later
};

__device__ __forceinline__ RowAddr row_addr(const StoreParams &p, uint32_t row, uint32_t &token) {
  const uint32_t plane = p.by_tokens.div(row);
  token = row - plane * p.by_tokens.d;
  const uint32_t layer = plane >> 1;
  RowAddr a;
  if (plane & 1u) {
    a.src = p.v + static_cast<int64_t>(layer) * p.v_layer_stride + static_cast<int64_t>(token) * p.v_row_stride;
    a.dst_base = p.v_cache + static_cast<int64_t>(layer) * p.cache_layer_stride;
  } else {
    a.src = p.k + static_cast<int64_t>(layer) * p.k_layer_stride + static_cast<int64_t>(token) * p.k_row_stride;
    a.dst_base = p.k_cache + static_cast<int64_t>(layer) * p.cache_layer_stride;
  }
  return a;
}

// Fast path: row = G lanes x VPL vectors x W bytes, R rows per group-iteration.
template <int W, int G, int VPL, int R, typename SlotT>
__global__ void __launch_bounds__(256) store_rows_kernel(const __grid_constant__ StoreParams p) {
  const uint32_t lane = threadIdx.x % G;
  const uint32_t group = (blockIdx.x * blockDim.x + threadIdx.x) / G;
  const uint32_t num_groups = (gridDim.x * blockDim.x) / G;

  for (uint32_t base = group * R; base < p.total_rows; base += num_groups * R) {
    Vec<W> data[R][VPL];
    char *dst[R];
    int64_t slot[R];
    bool live[R];
    // Issue every slot and row load of this iteration before consuming any.
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint32_t row = base + r;
      live[r] = row < p.total_rows;
      if (live[r]) {
        uint32_t token;
        const RowAddr a = row_addr(p, row, token);
        slot[r] = load_slot<SlotT>(p.slots, token);
        dst[r] = a.dst_base;
#pragma unroll
        for (int j = 0; j < VPL; ++j) load_vec(data[r][j], a.src + (j * G + lane) * W);
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (live[r]) {
        live[r] = slot_ok(slot[r], p);
        dst[r] += slot[r] * p.cache_row_stride;
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (live[r]) {
#pragma unroll
        for (int j = 0; j < VPL; ++j) store_vec(dst[r] + (j * G + lane) * W, data[r][j]);
      }
    }
  }
}

// Generic path: any row size and alignment, unit U in {1, 2, 4, 8, 16} bytes,
// one warp per row, four units in flight per lane.
template <typename U, typename SlotT>
__global__ void __launch_bounds__(256) store_rows_generic_kernel(const __grid_constant__ StoreParams p) {
  const uint32_t lane = threadIdx.x % 32;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const uint32_t num_warps = (gridDim.x * blockDim.x) / 32;
  for (uint32_t row = warp; row < p.total_rows; row += num_warps) {
    uint32_t token;
    const RowAddr a = row_addr(p, row, token);
    const int64_t slot = load_slot<SlotT>(p.slots, token);
    if (!slot_ok(slot, p)) continue;
    const U *src = reinterpret_cast<const U *>(a.src);
    U *dst = reinterpret_cast<U *>(a.dst_base + slot * p.cache_row_stride);
    for (uint32_t u = lane; u < p.row_units; u += 4 * 32) {
      U t[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t e = u + j * 32;
        if (e < p.row_units) t[j] = src[e];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t e = u + j * 32;
        if (e < p.row_units) dst[e] = t[j];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host side: pick a kernel for (row bytes, vector width, slot type), size the
// grid to the resident capacity of the device, launch.
// ---------------------------------------------------------------------------
using StoreKernel = void (*)(StoreParams);

struct StoreVariant {
  StoreKernel fn;
  int group;       // lanes per row
  int rows;        // rows per group-iteration
};

template <int W, int G, int VPL, int R>
StoreVariant make_variant(bool slot64) {
  return StoreVariant{slot64 ? store_rows_kernel<W, G, VPL, R, int64_t> : store_rows_kernel<W, G, VPL, R, int32_t>,
                      G, R};
}

// Vector width of the fast path: 16-byte vectors by default, 32-byte (v8)
// vectors when YL_STORE_VECTOR_BYTES=32 is set in the environment.
static int fast_vector_bytes() {
  static int w = [] {
    const char *e = std::getenv("YL_STORE_VECTOR_BYTES");
    return (e != nullptr && std::strcmp(e, "32") == 0) ? 32 : 16;
  }();
  return w;
}

static bool pick_fast(int64_t row_bytes, int w, bool slot64, StoreVariant &out) {
  if (w == 16) {
    switch (row_bytes) {
      case 16: out = make_variant<16, 1, 1, 8>(slot64); return true;
      case 32: out = make_variant<16, 2, 1, 8>(slot64); return true;
      case 64: out = make_variant<16, 4, 1, 8>(slot64); return true;
      case 128: out = make_variant<16, 8, 1, 8>(slot64); return true;
      case 256: out = make_variant<16, 16, 1, 8>(slot64); return true;
      case 512: out = make_variant<16, 32, 1, 8>(slot64); return true;
      case 1024: out = make_variant<16, 32, 2, 4>(slot64); return true;
      case 2048: out = make_variant<16, 32, 4, 2>(slot64); return true;
      case 4096: out = make_variant<16, 32, 8, 1>(slot64); return true;
      case 8192: out = make_variant<16, 32, 16, 1>(slot64); return true;
      default: return false;
    }
  }
  switch (row_bytes) {
    case 256: out = make_variant<32, 8, 1, 8>(slot64); return true;
    case 512: out = make_variant<32, 16, 1, 8>(slot64); return true;
    case 1024: out = make_variant<32, 32, 1, 4>(slot64); return true;
    case 2048: out = make_variant<32, 32, 2, 2>(slot64); return true;
    case 4096: out = make_variant<32, 32, 4, 1>(slot64); return true;
    case 8192: out = make_variant<32, 32, 8, 1>(slot64); return true;
    default: return false;
  }
}

static StoreVariant pick_generic(int unit, bool slot64) {
  StoreVariant v{nullptr, 32, 1};
  switch (unit) {
    case 16: v.fn = slot64 ? store_rows_generic_kernel<uint4, int64_t> : store_rows_generic_kernel<uint4, int32_t>; break;
    case 8: v.fn = slot64 ? store_rows_generic_kernel<uint2, int64_t> : store_rows_generic_kernel<uint2, int32_t>; break;
    case 4: v.fn = slot64 ? store_rows_generic_kernel<uint32_t, int64_t> : store_rows_generic_kernel<uint32_t, int32_t>; break;
    case 2: v.fn = slot64 ? store_rows_generic_kernel<uint16_t, int64_t> : store_rows_generic_kernel<uint16_t, int32_t>; break;
    default: v.fn = slot64 ? store_rows_generic_kernel<uint8_t, int64_t> : store_rows_generic_kernel<uint8_t, int32_t>; break;
  }
  return v;
}

static int widest_unit(uintptr_t bits) {
  for (int u = 16; u > 1; u >>= 1)
    if ((bits & static_cast<uintptr_t>(u - 1)) == 0) return u;
  return 1;
}

constexpr int kStoreThreads = 256;

// Resident blocks per SM of a store kernel on the current device (cached).
static int blocks_per_sm(StoreKernel fn) {
  static std::mutex mu;
  static std::map<std::pair<int, const void *>, int> cache;
  const std::pair<int, const void *> key{current_device(), reinterpret_cast<const void *>(fn)};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kStoreThreads, 0) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 1;
  }
  cache.emplace(key, n);
  return n;
}

}  // namespace ylk

extern "C" int yl_kv_store(const yl_store_args *a, cudaStream_t stream) {
  using namespace ylk;
  clear_last_error();
  if (a == nullptr) return fail(YL_ERR_NULL_ARG, "yl_kv_store: args is NULL");
  if (a->num_tokens < 0) return fail(YL_ERR_BAD_SIZE, "yl_kv_store: num_tokens=%lld < 0", a->num_tokens);
  if (a->num_layers < 1) return fail(YL_ERR_BAD_SIZE, "yl_kv_store: num_layers=%lld < 1", a->num_layers);
  if (a->row_bytes <= 0) return fail(YL_ERR_BAD_SIZE, "yl_kv_store: row_bytes=%lld <= 0", a->row_bytes);
  if (a->num_tokens == 0) return YL_OK;  // MHAKVCache::StoreKV returns early on N == 0
  if (!a->k || !a->v || !a->k_cache || !a->v_cache || !a->slots)
    return fail(YL_ERR_NULL_ARG, "yl_kv_store: k, v, k_cache, v_cache and slots must be non-NULL");
  if (a->slot_is_int64 != 0 && a->slot_is_int64 != 1)
    return fail(YL_ERR_BAD_SIZE, "yl_kv_store: slot_is_int64=%lld must be 0 or 1", a->slot_is_int64);
  if (a->k_row_stride < a->row_bytes || a->v_row_stride < a->row_bytes || a->cache_row_stride < a->row_bytes)
    return fail(YL_ERR_BAD_SIZE, "yl_kv_store: row strides must be >= row_bytes=%lld", a->row_bytes);
  const uint64_t total_rows = 2ull * static_cast<uint64_t>(a->num_layers) * static_cast<uint64_t>(a->num_tokens);
  if (total_rows >= (1ull << 31))
    return fail(YL_ERR_UNSUPPORTED, "yl_kv_store: 2*L*N=%lld rows exceeds 2^31-1 per call", (long long)total_rows);

  const bool multi = a->num_layers > 1;
  uintptr_t bits = reinterpret_cast<uintptr_t>(a->k) | reinterpret_cast<uintptr_t>(a->v) |
                   reinterpret_cast<uintptr_t>(a->k_cache) | reinterpret_cast<uintptr_t>(a->v_cache) |
                   static_cast<uintptr_t>(a->row_bytes) | static_cast<uintptr_t>(a->k_row_stride) |
                   static_cast<uintptr_t>(a->v_row_stride) | static_cast<uintptr_t>(a->cache_row_stride);
  if (multi)
    bits |= static_cast<uintptr_t>(a->k_layer_stride) | static_cast<uintptr_t>(a->v_layer_stride) |
            static_cast<uintptr_t>(a->cache_layer_stride);
  const int unit = widest_unit(bits);
  const size_t slot_bytes = a->slot_is_int64 ? 8 : 4;
  if ((reinterpret_cast<uintptr_t>(a->slots) & (slot_bytes - 1)) != 0)
    return fail(YL_ERR_ALIGNMENT, "yl_kv_store: slots pointer is not %lld-byte aligned", (long long)slot_bytes);

  StoreParams p;
  p.k = static_cast<const char *>(a->k);
  p.v = static_cast<const char *>(a->v);
  p.k_cache = static_cast<char *>(a->k_cache);
  p.v_cache = static_cast<char *>(a->v_cache);
  p.slots = a->slots;
  p.k_row_stride = a->k_row_stride;
  p.v_row_stride = a->v_row_stride;
  p.cache_row_stride = a->cache_row_stride;
  p.k_layer_stride = multi ? a->k_layer_stride : 0;
  p.v_layer_stride = multi ? a->v_layer_stride : 0;
  p.cache_layer_stride = multi ? a->cache_layer_stride : 0;
  p.num_slots = a->num_slots;
  p.error_word = a->error_word;
  p.total_rows = static_cast<uint32_t>(total_rows);
  p.row_units = static_cast<uint32_t>(a->row_bytes / unit);
  p.by_tokens = FastDiv(static_cast<uint32_t>(a->num_tokens));

  const bool slot64 = a->slot_is_int64 != 0;
  StoreVariant var{};
  bool fast = false;
  const int w = fast_vector_bytes();
  if (unit == 16 && w == 32 && ((bits & 31u) == 0)) fast = pick_fast(a->row_bytes, 32, slot64, var);
  if (!fast && unit == 16) fast = pick_fast(a->row_bytes, 16, slot64, var);
  if (!fast) {
    if (a->row_bytes / unit >= (1ll << 31))
      return fail(YL_ERR_UNSUPPORTED, "yl_kv_store: row_bytes=%lld too large", a->row_bytes);
    var = pick_generic(unit, slot64);
  }

  const uint64_t rows_per_block = static_cast<uint64_t>(kStoreThreads / var.group) * var.rows;
  const uint64_t want = (total_rows + rows_per_block - 1) / rows_per_block;
  const uint64_t cap = static_cast<uint64_t>(sm_count()) * blocks_per_sm(var.fn);
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  var.fn<<<grid, kStoreThreads, 0, stream>>>(p);
  return check_launch("yl_kv_store launch");
}
