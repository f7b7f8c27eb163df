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
#include <string>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>
#include <vector>

#include "common.cuh"
#include "store_device.cuh"
#include "tma.cuh"

namespace ylk {

// Fast path: row = G lanes x VPL vectors x W bytes, R rows per group-iteration.
template <int W, int G, int VPL, int R, typename SlotT>
__global__ void __launch_bounds__(256) store_rows_kernel(const __grid_constant__ StoreParams p) {
  const uint32_t lane = threadIdx.x % G;
  const uint32_t group = (blockIdx.x * blockDim.x + threadIdx.x) / G;
  const uint32_t num_groups = (gridDim.x * blockDim.x) / G;

  uint32_t base = group * R;
  RowBatch<W, G, VPL, R> b;
  b.load(p, base, lane);
  // The K/V rows are in flight; the slots may be written by the kernel just
  // before this one (the index build, when launched as its PDL dependent).
  pdl_wait();
  while (base < p.total_rows) {
    int64_t slot[R];
#pragma unroll
    for (int r = 0; r < R; ++r) slot[r] = b.live[r] ? load_slot<SlotT>(p.slots, b.token[r]) : -1;
#pragma unroll
    for (int r = 0; r < R; ++r) b.resolve(p, r, slot[r]);
    b.store(lane);
    base += num_groups * R;
    if (base < p.total_rows) b.load(p, base, lane);
  }
}

// A decode step's store, token by token.  Work unit u = (plane chunk c,
// token t), u = c * N + t, one unit per lane group: the group computes its
// token's slot once (or reads it, for a batch that is not a decode batch),
// then copies the token's rows of planes [c * chunk, (c + 1) * chunk), R
// planes in flight at a time, stepping its source and destination rows by the
// layer strides (no per-row division or slot lookup, which for small rows
// costs more issue slots than the copy).  Consecutive groups take consecutive
// tokens of the same planes, so the K/V reads of a warp are contiguous.
template <int W, int G, int VPL, int R, typename SlotT>
__global__ void __launch_bounds__(256) store_decode_kernel(const __grid_constant__ StoreParams p, uint32_t chunk,
                                                           uint32_t planes) {
  const uint32_t lane = threadIdx.x % G;
  const uint32_t unit = (blockIdx.x * blockDim.x + threadIdx.x) / G;
  const uint32_t N = p.by_tokens.d;
  const uint32_t c = p.by_tokens.div(unit);
  const uint32_t t = unit - c * N;
  uint32_t pl = c * chunk;
  const uint32_t end = min(pl + chunk, planes);
  const char *src_k = p.k + static_cast<int64_t>(t) * p.k_row_stride;
  const char *src_v = p.v + static_cast<int64_t>(t) * p.v_row_stride;
  Vec<W> data[R][VPL];
  auto load = [&](uint32_t first) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint32_t q = first + r;
      if (q < end) {
        const int64_t layer = q >> 1;
        const char *src = (q & 1u) ? src_v + layer * p.v_layer_stride : src_k + layer * p.k_layer_stride;
#pragma unroll
        for (int j = 0; j < VPL; ++j) load_vec(data[r][j], src + (j * G + lane) * W);
      }
    }
  };
  load(pl);
  const bool self = decode_batch(p.self);  // block-uniform
  int64_t slot = -1;
  if (!self) {
    pdl_wait();
    if (pl < end) slot = load_slot<SlotT>(p.slots, t);
  } else if (pl < end) {
    slot = decode_slot(p.self, t, p.error_word);
  }
  const bool ok = pl < end && slot_ok(slot, p);
  char *dst_k = p.k_cache + slot * p.cache_row_stride;
  char *dst_v = p.v_cache + slot * p.cache_row_stride;
  while (pl < end) {
    if (ok) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t q = pl + r;
        if (q < end) {
          char *dst = ((q & 1u) ? dst_v : dst_k) + static_cast<int64_t>(q >> 1) * p.cache_layer_stride;
#pragma unroll
          for (int j = 0; j < VPL; ++j) store_vec(dst + (j * G + lane) * W, data[r][j]);
        }
      }
    }
    pl += R;
    if (pl < end) load(pl);
  }
  // Computing its own slots, this grid never waited for the index build it
  // was launched behind; wait before exiting, so that its completion implies
  // the index build's (a kernel launched as its programmatic dependent, such
  // as the next step's index build, relies on that order).
  if (self) pdl_wait();
}

// TMA path: one CTA per SM stages its rows in shared memory.  The CTA owns a
// contiguous range of rows; a round loads up to nslot of them with bulk
// copies (thread t owns stage slots t, t + 256, ...), so at kernel start
// nearly all of a decode step's K/V reads are in flight before the kernel
// waits for its slots (pdl_wait, when launched behind the index build).  Once
// a thread's rows have landed and their slots are known it bulk-stores them
// from shared memory and, when the next round needs its stage slots, waits
// only until those stores have read shared memory.
constexpr int kTmaThreads = 256;
constexpr int kTmaSlotsPerThread = 8;
constexpr uint64_t kTmaWaitLimitNs = kBulkWaitLimitNs;  // 2 s
constexpr size_t kTmaBarrierBytes = kTmaThreads * sizeof(uint64_t);

template <typename SlotT>
__global__ void __launch_bounds__(kTmaThreads, 1)
    store_rows_tma_kernel(const __grid_constant__ StoreParams p, uint32_t row_bytes, uint32_t nslot,
                          uint32_t rows_per_cta) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem_raw) + threadIdx.x;
  char *stage = reinterpret_cast<char *>(smem_raw) + kTmaBarrierBytes;
  const uint32_t begin = blockIdx.x * rows_per_cta;
  const uint32_t end = min(begin + rows_per_cta, p.total_rows);
  mbar_init(bar, 1);  // each thread waits only on its own barrier
  fence_mbar_init();

  // Issue round r's loads; false when this thread has no row in it.
  auto issue = [&](uint32_t r) -> bool {
    const uint32_t first = begin + r * nslot;
    uint32_t bytes = 0;
#pragma unroll
    for (int k = 0; k < kTmaSlotsPerThread; ++k) {
      const uint32_t sl = threadIdx.x + k * kTmaThreads;
      if (sl < nslot && first + sl < end) bytes += row_bytes;
    }
    if (bytes == 0) return false;
    mbar_arrive_expect_tx(bar, bytes);
#pragma unroll
    for (int k = 0; k < kTmaSlotsPerThread; ++k) {
      const uint32_t sl = threadIdx.x + k * kTmaThreads;
      if (sl < nslot && first + sl < end) {
        uint32_t token;
        const RowAddr a = row_addr(p, first + sl, token);
        bulk_load(stage + static_cast<size_t>(sl) * row_bytes, a.src, row_bytes, bar);
      }
    }
    return true;
  };

  uint32_t r = 0, parity = 0;
  bool have = issue(0);
  pdl_wait();  // slots may come from the kernel this one was launched behind
  while (have) {
    const uint32_t first = begin + r * nslot;
    int64_t slot[kTmaSlotsPerThread];
#pragma unroll
    for (int k = 0; k < kTmaSlotsPerThread; ++k) {
      const uint32_t sl = threadIdx.x + k * kTmaThreads;
      slot[k] = -1;
      if (sl < nslot && first + sl < end) {
        const uint32_t plane = p.by_tokens.div(first + sl);
        slot[k] = load_slot<SlotT>(p.slots, first + sl - plane * p.by_tokens.d);
      }
    }
    if (!mbar_wait_bounded(bar, parity, p.wait_limit_ns)) {
      raise_deverr(p.error_word, YL_DEVERR_TIMEOUT);
      mbar_wait_bounded(bar, parity, kTmaWaitLimitNs);  // let this thread's loads land before leaving
      break;
    }
#pragma unroll
    for (int k = 0; k < kTmaSlotsPerThread; ++k) {
      const uint32_t sl = threadIdx.x + k * kTmaThreads;
      if (sl < nslot && first + sl < end && slot_ok(slot[k], p)) {
        uint32_t token;
        const RowAddr a = row_addr(p, first + sl, token);
        bulk_store(a.dst_base + slot[k] * p.cache_row_stride, stage + static_cast<size_t>(sl) * row_bytes,
                   row_bytes);
      }
    }
    bulk_commit();
    ++r;
    parity ^= 1u;
    if (begin + r * nslot >= end) break;
    bulk_wait_read_all();  // this thread's stage slots are free again
    have = issue(r);
  }
  bulk_wait_all();
}

// Generic path: any row size and alignment, unit U in {1, 2, 4, 8, 16} bytes,
// one warp per row, four units in flight per lane.
template <typename U, typename SlotT>
__global__ void __launch_bounds__(256) store_rows_generic_kernel(const __grid_constant__ StoreParams p) {
  const uint32_t lane = threadIdx.x % 32;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const uint32_t num_warps = (gridDim.x * blockDim.x) / 32;
  pdl_wait();
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
// Host side: validate, pick a kernel for (row bytes, vector width, slot type),
// size the grid to the resident capacity of the device, launch.
// ---------------------------------------------------------------------------
using StoreKernel = void (*)(StoreParams);

using DecodeKernel = void (*)(StoreParams, uint32_t, uint32_t);
constexpr uint64_t kDecodeUnitBytes = 20 * 1024;  // rows one lane group of the decode store takes at most
struct StoreVariant {
  StoreKernel fn;
  int group;  // lanes per row
  int rows;   // rows per group-iteration
  DecodeKernel dec = nullptr;  // the decode step's token-by-token kernel (fn unused)
};

int fast_vector_bytes() {
  static int w = [] {
    const char *e = std::getenv("YL_STORE_VECTOR_BYTES");
    return (e != nullptr && std::strcmp(e, "16") == 0) ? 16 : 32;
  }();
  return w;
}

// self: the decode step's token-by-token store (store_decode_kernel), else
// the plain store.
static bool pick_fast(int64_t row_bytes, int w, bool slot64, bool self, StoreVariant &out) {
  return dispatch_row_shape(row_bytes, w, [&](auto shape) {
    using S = decltype(shape);
    // The decode store keeps at most 4 rows in flight per lane group: for
    // 256-512-byte rows the store's 8 (102 registers, 2 CTAs per SM) leave
    // no registers for the index build beside it, whose blocks then hold
    // half of each SM's store CTAs back (one rank at 8 GPUs: 20.4 -> 18.8 us
    // per step; Qwen2-72B decode at one head per GPU: 13.6 -> 11.6 us).
    constexpr int RD = S::R > 4 ? 4 : S::R;
    if (self)
      out = StoreVariant{nullptr, S::G, RD,
                         slot64 ? store_decode_kernel<S::W, S::G, S::VPL, RD, int64_t>
                                : store_decode_kernel<S::W, S::G, S::VPL, RD, int32_t>};
    else
      out = StoreVariant{slot64 ? store_rows_kernel<S::W, S::G, S::VPL, S::R, int64_t>
                                : store_rows_kernel<S::W, S::G, S::VPL, S::R, int32_t>,
                         S::G, S::R};
  });
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

// Resident blocks per SM of a kernel at kStoreThreads threads (cached per device).
int blocks_per_sm(const void *fn, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void *, size_t>, int> cache;
  const auto key = std::make_tuple(current_device(), fn, smem);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kStoreThreads, smem) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 1;
  }
  cache.emplace(key, n);
  return n;
}

int prepare_store(const yl_store_args *a, bool need_slots, StorePlan &plan) {
  if (a == nullptr) return fail(YL_ERR_NULL_ARG, "yl_kv_store: args is NULL");
  if (a->num_tokens < 0) return fail(YL_ERR_BAD_SIZE, "yl_kv_store: num_tokens=%lld < 0", a->num_tokens);
  if (a->num_layers < 1) return fail(YL_ERR_BAD_SIZE, "yl_kv_store: num_layers=%lld < 1", a->num_layers);
  if (a->row_bytes <= 0) return fail(YL_ERR_BAD_SIZE, "yl_kv_store: row_bytes=%lld <= 0", a->row_bytes);
  if (a->num_tokens == 0) return YL_OK;  // MHAKVCache::StoreKV returns early on N == 0
  if (!a->k || !a->v || !a->k_cache || !a->v_cache || (need_slots && !a->slots))
    return fail(YL_ERR_NULL_ARG, "yl_kv_store: k, v, k_cache, v_cache and slots must be non-NULL");
  if (a->slot_is_int64 != 0 && a->slot_is_int64 != 1)
    return fail(YL_ERR_BAD_SIZE, "yl_kv_store: slot_is_int64=%lld must be 0 or 1", a->slot_is_int64);
  if (a->k_row_stride < a->row_bytes || a->v_row_stride < a->row_bytes || a->cache_row_stride < a->row_bytes)
    return fail(YL_ERR_BAD_SIZE, "yl_kv_store: row strides must be >= row_bytes=%lld", a->row_bytes);
  const uint64_t total_rows = 2ull * static_cast<uint64_t>(a->num_layers) * static_cast<uint64_t>(a->num_tokens);
  if (total_rows >= (1ull << 31))
    return fail(YL_ERR_UNSUPPORTED, "yl_kv_store: 2*L*N=%lld rows exceeds 2^31-1 per call", (long long)total_rows);
  const size_t slot_bytes = a->slot_is_int64 ? 8 : 4;
  if (need_slots && (reinterpret_cast<uintptr_t>(a->slots) & (slot_bytes - 1)) != 0)
    return fail(YL_ERR_ALIGNMENT, "yl_kv_store: slots pointer is not %lld-byte aligned", (long long)slot_bytes);

  const bool multi = a->num_layers > 1;
  uintptr_t bits = reinterpret_cast<uintptr_t>(a->k) | reinterpret_cast<uintptr_t>(a->v) |
                   reinterpret_cast<uintptr_t>(a->k_cache) | reinterpret_cast<uintptr_t>(a->v_cache) |
                   static_cast<uintptr_t>(a->row_bytes) | static_cast<uintptr_t>(a->k_row_stride) |
                   static_cast<uintptr_t>(a->v_row_stride) | static_cast<uintptr_t>(a->cache_row_stride);
  if (multi)
    bits |= static_cast<uintptr_t>(a->k_layer_stride) | static_cast<uintptr_t>(a->v_layer_stride) |
            static_cast<uintptr_t>(a->cache_layer_stride);
  plan.bits = bits;
  plan.unit = widest_unit(bits);
  if (a->row_bytes / plan.unit >= (1ll << 31))
    return fail(YL_ERR_UNSUPPORTED, "yl_kv_store: row_bytes=%lld too large", a->row_bytes);

  StoreParams &p = plan.p;
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
  p.self = SelfSlots{};
  p.total_rows = static_cast<uint32_t>(total_rows);
  p.row_units = static_cast<uint32_t>(a->row_bytes / plan.unit);
  p.by_tokens = FastDiv(static_cast<uint32_t>(a->num_tokens));
  p.wait_limit_ns = bulk_wait_limit_ns();
  return YL_OK;
}

// Store engine: register-staged vector copies (default) or TMA bulk copies
// staged in shared memory (YL_STORE_ENGINE=tma).
static bool use_tma_engine() {
  static const bool t = [] {
    const char *e = std::getenv("YL_STORE_ENGINE");
    return e != nullptr && std::strcmp(e, "tma") == 0;
  }();
  return t;
}

// Staging per CTA: 200 KB of the SM's 228 KB, leaving room for two index-build
// blocks to stay resident beside it when the store runs as their PDL dependent.
constexpr size_t kTmaMaxSmem = 200 * 1024;

static int launch_store_tma(const StorePlan &plan, int64_t row_bytes, bool slot64, cudaStream_t stream, bool pdl) {
  using TmaKernel = void (*)(StoreParams, uint32_t, uint32_t, uint32_t);
  const TmaKernel fn = slot64 ? store_rows_tma_kernel<int64_t> : store_rows_tma_kernel<int32_t>;
  static std::mutex mu;
  static std::vector<char> done;
  {
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(done.size()) <= dev) done.resize(dev + 1, 0);
    if (!(done[dev] & (slot64 ? 2 : 1))) {
      cudaError_t e =
          cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTmaMaxSmem));
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) {
        cudaGetLastError();
        set_last_error(std::string("yl_kv_store: cudaFuncSetAttribute: ") + cudaGetErrorString(e));
        return YL_ERR_CUDA;
      }
      done[dev] |= (slot64 ? 2 : 1);
    }
  }
  const uint64_t cap_slots = (kTmaMaxSmem - kTmaBarrierBytes) / static_cast<uint64_t>(row_bytes);
  const uint32_t nslot = static_cast<uint32_t>(
      cap_slots < static_cast<uint64_t>(kTmaThreads * kTmaSlotsPerThread) ? cap_slots : kTmaThreads * kTmaSlotsPerThread);
  const uint64_t total = plan.p.total_rows;
  uint64_t grid = (total + 63) / 64;
  const uint64_t sms = static_cast<uint64_t>(sm_count());
  if (grid > sms) grid = sms;
  if (grid < 1) grid = 1;
  const uint32_t rows_per_cta = static_cast<uint32_t>((total + grid - 1) / grid);
  const uint64_t per_round = rows_per_cta < nslot ? rows_per_cta : nslot;
  const size_t smem = kTmaBarrierBytes + static_cast<size_t>(per_round) * static_cast<size_t>(row_bytes);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kTmaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, plan.p, static_cast<uint32_t>(row_bytes),
                                           static_cast<uint32_t>(per_round), rows_per_cta);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_last_error(std::string("yl_kv_store launch: ") + cudaGetErrorString(e));
    return YL_ERR_CUDA;
  }
  return check_launch("yl_kv_store launch");
}

int launch_store(const StorePlan &plan, int64_t row_bytes, bool slot64, cudaStream_t stream, bool pdl) {
  if (use_tma_engine() && plan.unit == 16 && row_bytes <= 16384) return launch_store_tma(plan, row_bytes, slot64, stream, pdl);
  StoreVariant var{};
  bool fast = false;
  const int w = fast_vector_bytes();
  const bool self = plan.p.self.batch > 0;
  if (plan.unit == 16 && w == 32 && (plan.bits & 31u) == 0) fast = pick_fast(row_bytes, 32, slot64, self, var);
  if (!fast && plan.unit == 16) fast = pick_fast(row_bytes, 16, slot64, self, var);
  if (!fast) var = pick_generic(plan.unit, slot64);  // reads the slots after the index build (pdl_wait)
  const uint64_t rows_per_block = static_cast<uint64_t>(kStoreThreads / var.group) * var.rows;
  const uint64_t want = (plan.p.total_rows + rows_per_block - 1) / rows_per_block;
  if (var.dec != nullptr) {
    // units of (plane chunk, token): chunks of R-plane multiples sized so
    // that the resident lane groups of one wave take every unit, at most 4R
    const uint64_t n = plan.p.by_tokens.d;
    const uint64_t planes = plan.p.total_rows / n;
    const uint64_t groups = kStoreThreads / var.group;
    const uint64_t R = static_cast<uint64_t>(var.rows);
    const uint64_t resident = static_cast<uint64_t>(sm_count()) *
                              blocks_per_sm(reinterpret_cast<const void *>(var.dec), 0) * groups;
    uint64_t chunk = R * ((planes * n + resident * R - 1) / (resident * R));
    // at most kDecodeUnitBytes of rows per unit: in a long store (80 layers)
    // the CTAs that start late, behind the index build's blocks, would
    // otherwise carry long runs past everyone else (Qwen2-72B decode, 8 heads:
    // 60.8 -> ~58 us per step with 10-plane runs of 2 KB rows instead of 18;
    // a 32-layer decode step keeps its 4-plane runs, Qwen2-72B at 4 heads per
    // GPU its 20 planes of 1 KB)
    const uint64_t cap_planes = kDecodeUnitBytes / static_cast<uint64_t>(row_bytes) / R * R;
    if (cap_planes >= R && chunk > cap_planes) chunk = cap_planes;
    const uint64_t max_chunk = (planes + R - 1) / R * R;
    if (chunk > max_chunk) chunk = max_chunk;
    const uint64_t units = (planes + chunk - 1) / chunk * n;
    const unsigned grid = static_cast<unsigned>((units + groups - 1) / groups);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kStoreThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, var.dec, plan.p, static_cast<uint32_t>(chunk),
                                             static_cast<uint32_t>(planes));
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_last_error(std::string("yl_kv_store launch: ") + cudaGetErrorString(e));
      return YL_ERR_CUDA;
    }
    return YL_OK;
  }
  const size_t smem = 0;
  const uint64_t cap =
      static_cast<uint64_t>(sm_count()) * blocks_per_sm(reinterpret_cast<const void *>(var.fn), smem);
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kStoreThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, var.fn, plan.p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_last_error(std::string("yl_kv_store launch: ") + cudaGetErrorString(e));
    return YL_ERR_CUDA;
  }
  return check_launch("yl_kv_store launch");
}

}  // namespace ylk

extern "C" int yl_kv_store(const yl_store_args *a, cudaStream_t stream) {
  using namespace ylk;
  clear_last_error();
  StorePlan plan;
  const int rc = prepare_store(a, true, plan);
  if (rc != YL_OK || a->num_tokens == 0) return rc;
  return launch_store(plan, a->row_bytes, a->slot_is_int64 != 0, stream, false);
}
