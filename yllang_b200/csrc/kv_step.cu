// One serving step of the path in one launch: the batch index build followed
// by the store of every layer's new K/V rows under the slot mapping it
// produces (yl_build_index then yl_kv_store, fused).
//
// Why fused on B200: at decode sizes the store moves ~67 MB (Llama-3-8B
// shape, 256 sequences) — about 10 us of HBM time — so a separate index
// launch, its dependent global round trips, and a second launch's ramp and
// drain cost as much as the copy.  Here every block first issues the loads of
// its first K/V rows (they do not depend on the index), then computes the
// batch scan in shared memory while those loads are in flight, writes its
// share of the page arrays, and derives each row's slot on the fly from the
// scanned offsets and the page table; the rows of layer 0's K plane also
// write slot_mapping.  Batches above kStepBatchLimit sequences, or rows
// without a 16-byte fast shape, run as the two separate launches instead.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "index_device.cuh"
#include "store_device.cuh"
#include "tma.cuh"

namespace ylk {

struct StepParams {
  IndexParams ix;
  StoreParams st;
  uint32_t num_tokens;  // N, rows per plane
};

constexpr int kStepThreads = 256;
constexpr int kStepBatchLimit = 4096;
// Three resident blocks per SM: the K/V rows of the first iteration stay in
// registers across the scan, and 3 x 256 threads keep ~100 KB of row loads in
// flight per SM for 2 KB rows without spilling.

int blocks_per_sm(const void *fn, size_t smem);  // kv_store.cu, at 256 threads

template <int W, int G, int VPL, int R>
__global__ void __launch_bounds__(kStepThreads, 3) kv_step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ int64_t smem[];
  int64_t *scratch = smem;                                // kScanScratch x int64
  int32_t *kvp = reinterpret_cast<int32_t *>(smem + kScanScratch);  // [B+1]
  int32_t *qop = kvp + (p.ix.batch + 1);                  // [B+1]
  const uint32_t lane = threadIdx.x % G;
  const uint32_t group = (blockIdx.x * blockDim.x + threadIdx.x) / G;
  const uint32_t num_groups = (gridDim.x * blockDim.x) / G;
  const bool report = blockIdx.x == 0;

  // The K/V rows of the first iteration do not depend on the index build.
  uint32_t base = group * R;
  RowBatch<W, G, VPL, R> b;
  b.load(p.st, base, lane);

  if (!scan_batch(p.ix, kvp, qop, scratch, report)) return;  // uniform per block
  const int64_t n_tok = qop[p.ix.batch];
  if (report && threadIdx.x == 0 && n_tok != p.num_tokens) raise_deverr(p.ix.error_word, YL_DEVERR_TOKEN_COUNT);
  write_seq_outputs(p.ix, kvp, qop, static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x,
                    static_cast<int64_t>(gridDim.x) * blockDim.x, true);
  fill_kv_share(p.ix, kvp, p.num_tokens, report);

  for (;;) {
    int64_t slot[R];
#pragma unroll
    for (int r = 0; r < R; ++r)
      slot[r] = (b.live[r] && b.token[r] < n_tok) ? token_slot(p.ix, kvp, qop, b.token[r]) : -1;
#pragma unroll
    for (int r = 0; r < R; ++r)  // rows of plane 0 (layer 0, K) publish the slot mapping
      if (b.live[r] && base + r < p.num_tokens && lane == 0) write_slot(p.ix, b.token[r], slot[r]);
#pragma unroll
    for (int r = 0; r < R; ++r) b.resolve(p.st, r, slot[r]);
    b.store(lane);
    base += num_groups * R;
    if (base >= p.st.total_rows) break;
    b.load(p.st, base, lane);
  }
}

// TMA-staged fused step.  One CTA per SM owns a contiguous range of rows and
// stages them in shared memory: at kernel start every staging thread
// (threads own stage slots t, t + 256, ...) issues bulk loads of its rows, so
// for a decode step all of the step's K/V reads are in flight from the first
// microsecond.  While they land, all threads compute the batch scan and this
// CTA's share of the page arrays; then each staging thread derives its rows'
// slots, waits for its rows, and bulk-stores them to the pool.
constexpr int kTmaSlotsPerThread = 8;
constexpr uint64_t kTmaWaitLimitNs = kBulkWaitLimitNs;  // 2 s
constexpr size_t kTmaSmemMax = 232448;               // 227 KB, the B200 per-CTA maximum

static size_t tma_header_bytes(int batch) {
  const size_t h = kStepThreads * sizeof(uint64_t) + kScanScratch * sizeof(int64_t) + 2 * (batch + 1) * sizeof(int32_t);
  return (h + 127) & ~static_cast<size_t>(127);
}

__global__ void __launch_bounds__(kStepThreads, 1)
    kv_step_tma_kernel(const __grid_constant__ StepParams p, uint32_t row_bytes, uint32_t nslot,
                       uint32_t rows_per_cta, uint32_t header) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem_raw) + threadIdx.x;
  int64_t *scratch = reinterpret_cast<int64_t *>(smem_raw + kStepThreads * sizeof(uint64_t));
  int32_t *kvp = reinterpret_cast<int32_t *>(scratch + kScanScratch);
  int32_t *qop = kvp + (p.ix.batch + 1);
  char *stage = reinterpret_cast<char *>(smem_raw) + header;
  const StoreParams &st = p.st;
  const uint32_t begin = blockIdx.x * rows_per_cta;
  const uint32_t end = min(begin + rows_per_cta, st.total_rows);
  const bool report = blockIdx.x == 0;
  mbar_init(bar, 1);  // each thread waits only on its own barrier
  fence_mbar_init();

  auto issue = [&](uint32_t r) -> bool {
    const uint32_t first = begin + r * nslot;
    uint32_t bytes = 0;
#pragma unroll
    for (int k = 0; k < kTmaSlotsPerThread; ++k) {
      const uint32_t sl = threadIdx.x + k * kStepThreads;
      if (sl < nslot && first + sl < end) bytes += row_bytes;
    }
    if (bytes == 0) return false;
    mbar_arrive_expect_tx(bar, bytes);
#pragma unroll
    for (int k = 0; k < kTmaSlotsPerThread; ++k) {
      const uint32_t sl = threadIdx.x + k * kStepThreads;
      if (sl < nslot && first + sl < end) {
        uint32_t token;
        const RowAddr a = row_addr(st, first + sl, token);
        bulk_load(stage + static_cast<size_t>(sl) * row_bytes, a.src, row_bytes, bar);
      }
    }
    return true;
  };

  uint32_t r = 0, parity = 0;
  bool have = issue(0);  // the step's K/V reads start now

  if (!scan_batch(p.ix, kvp, qop, scratch, report)) {  // uniform per block
    if (have) mbar_wait_bounded(bar, parity, kTmaWaitLimitNs);  // let the loads land before leaving
    return;
  }
  const int64_t n_tok = qop[p.ix.batch];
  if (report && threadIdx.x == 0 && n_tok != p.num_tokens) raise_deverr(p.ix.error_word, YL_DEVERR_TOKEN_COUNT);
  write_seq_outputs(p.ix, kvp, qop, static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x,
                    static_cast<int64_t>(gridDim.x) * blockDim.x, true);
  fill_kv_share(p.ix, kvp, p.num_tokens, report);

  while (have) {
    const uint32_t first = begin + r * nslot;
    int64_t slot[kTmaSlotsPerThread];
#pragma unroll
    for (int k = 0; k < kTmaSlotsPerThread; ++k) {
      const uint32_t sl = threadIdx.x + k * kStepThreads;
      slot[k] = -1;
      if (sl < nslot && first + sl < end) {
        const uint32_t row = first + sl;
        const uint32_t plane = st.by_tokens.div(row);
        const uint32_t token = row - plane * st.by_tokens.d;
        if (token < n_tok) slot[k] = token_slot(p.ix, kvp, qop, token);
        if (plane == 0) write_slot(p.ix, token, slot[k]);  // layer 0's K rows publish the slot mapping
      }
    }
    if (!mbar_wait_bounded(bar, parity, st.wait_limit_ns)) {
      raise_deverr(p.ix.error_word, YL_DEVERR_TIMEOUT);
      mbar_wait_bounded(bar, parity, kTmaWaitLimitNs);  // let this thread's loads land before leaving
      break;
    }
#pragma unroll
    for (int k = 0; k < kTmaSlotsPerThread; ++k) {
      const uint32_t sl = threadIdx.x + k * kStepThreads;
      if (sl < nslot && first + sl < end && slot_ok(slot[k], st)) {
        uint32_t token;
        const RowAddr a = row_addr(st, first + sl, token);
        bulk_store(a.dst_base + slot[k] * st.cache_row_stride, stage + static_cast<size_t>(sl) * row_bytes,
                   row_bytes);
      }
    }
    bulk_commit();
    ++r;
    parity ^= 1u;
    if (begin + r * nslot >= end) break;
    bulk_wait_read_all();
    have = issue(r);
  }
  bulk_wait_all();
}

static size_t step_smem(int batch) { return kScanScratch * sizeof(int64_t) + 2 * (batch + 1) * sizeof(int32_t); }

// How yl_kv_step runs (YL_STEP_MODE): the index build and a PDL-dependent
// store (default, "pdl"), the TMA-staged fused kernel ("tma"), the
// register-staged fused kernel ("fused"), or the two launches serialised
// ("serial").  On B200 the PDL form is the fastest measured: the store's
// first K/V loads overlap the index build without tying up registers or
// shared memory across it.
enum class StepMode { kPdl, kTma, kFused, kSerial };

// Decode batches up to kStepSelfSlotsBatch sequences have the store compute
// their slots (store_decode_kernel: one slot per lane group and token).
constexpr int kStepSelfSlotsBatch = 16384;
static StepMode step_mode() {
  static const StepMode m = [] {
    const char *e = std::getenv("YL_STEP_MODE");
    if (e != nullptr && std::strcmp(e, "fused") == 0) return StepMode::kFused;
    if (e != nullptr && std::strcmp(e, "serial") == 0) return StepMode::kSerial;
    if (e != nullptr && std::strcmp(e, "tma") == 0) return StepMode::kTma;
    return StepMode::kPdl;
  }();
  return m;
}

static int launch_step_tma(const StepParams &p, int64_t row_bytes, cudaStream_t stream) {
  static std::mutex mu;
  static std::vector<char> done;
  {
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(done.size()) <= dev) done.resize(dev + 1, 0);
    if (!done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kv_step_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(kTmaSmemMax));
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kv_step_tma_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) {
        cudaGetLastError();
        set_last_error(std::string("yl_kv_step: cudaFuncSetAttribute: ") + cudaGetErrorString(e));
        return YL_ERR_CUDA;
      }
      done[dev] = 1;
    }
  }
  const size_t header = tma_header_bytes(p.ix.batch);
  const uint64_t cap = (kTmaSmemMax - header) / static_cast<uint64_t>(row_bytes);
  const uint64_t max_slots = static_cast<uint64_t>(kStepThreads) * kTmaSlotsPerThread;
  const uint64_t nslot_cap = cap < max_slots ? cap : max_slots;
  const uint64_t total = p.st.total_rows;
  // one CTA per SM, each with enough rows to fill its stage or a fair share
  uint64_t grid = static_cast<uint64_t>(sm_count());
  const uint64_t by_rows = (total + 31) / 32;
  if (by_rows < grid) grid = by_rows;
  const uint64_t fill = static_cast<uint64_t>(p.ix.indices_cap);
  const uint64_t by_fill = (fill + 4 * kStepThreads - 1) / (4 * kStepThreads);
  if (by_fill > grid) grid = by_fill < static_cast<uint64_t>(sm_count()) ? by_fill : sm_count();
  if (grid < 1) grid = 1;
  const uint32_t rows_per_cta = static_cast<uint32_t>((total + grid - 1) / grid);
  const uint32_t nslot = static_cast<uint32_t>(rows_per_cta < nslot_cap ? rows_per_cta : nslot_cap);
  const size_t smem = header + static_cast<size_t>(nslot) * static_cast<size_t>(row_bytes);
  kv_step_tma_kernel<<<static_cast<unsigned>(grid), kStepThreads, smem, stream>>>(
      p, static_cast<uint32_t>(row_bytes), nslot, rows_per_cta, static_cast<uint32_t>(header));
  return check_launch("yl_kv_step launch");
}

}  // namespace ylk

extern "C" int yl_kv_step(const yl_step_args *a, cudaStream_t stream) {
  using namespace ylk;
  clear_last_error();
  if (a == nullptr) return fail(YL_ERR_NULL_ARG, "yl_kv_step: args is NULL");
  IndexParams ix;
  int rc = prepare_index(&a->index, ix);
  if (rc != YL_OK) return rc;
  if (a->index.slot_mapping == nullptr) return fail(YL_ERR_NULL_ARG, "yl_kv_step: index.slot_mapping is required");
  if (a->store.num_tokens > a->index.slot_capacity)
    return fail(YL_ERR_BAD_SIZE, "yl_kv_step: num_tokens=%lld exceeds slot_capacity=%lld", a->store.num_tokens,
                a->index.slot_capacity);
  yl_store_args s = a->store;
  s.slots = a->index.slot_mapping;
  s.slot_is_int64 = a->index.slot_is_int64;
  s.error_word = a->index.error_word;
  StorePlan sp;
  rc = prepare_store(&s, true, sp);
  if (rc != YL_OK) return rc;
  ix.expected_tokens = s.num_tokens;
  if (s.num_tokens == 0) return launch_index(ix, stream);

  const int w = fast_vector_bytes();
  using StepKernel = void (*)(StepParams);
  StepKernel fn = nullptr;
  int group = 32, rows = 1;
  auto pick = [&](auto shape) {
    using S = decltype(shape);
    fn = kv_step_kernel<S::W, S::G, S::VPL, S::R>;
    group = S::G;
    rows = S::R;
  };
  bool fused = ix.batch <= kStepBatchLimit && sp.unit == 16;
  if (fused && step_mode() == StepMode::kTma && s.row_bytes <= 16384) {
    StepParams p;
    p.ix = ix;
    p.st = sp.p;
    p.num_tokens = static_cast<uint32_t>(s.num_tokens);
    return launch_step_tma(p, s.row_bytes, stream);
  }
  if (fused) {
    bool found = false;
    if (w == 32 && (sp.bits & 31u) == 0) found = dispatch_row_shape(s.row_bytes, 32, pick);
    if (!found) found = dispatch_row_shape(s.row_bytes, 16, pick);
    fused = found;
  }
  if (!fused || step_mode() == StepMode::kPdl || step_mode() == StepMode::kSerial) {
    // Two launches: the index build, then the store reading its slot mapping.
    // In PDL mode the store is the index kernel's programmatic dependent: its
    // K/V loads overlap the index build and only the slot reads wait for it.
    // A decode batch (N == B, and the store checks every new_len is 1) lets
    // the store compute its slots itself and run beside the index build
    // instead of after it: store_decode_kernel gives each lane group one
    // token, whose slot it computes once, and a run of that token's layers,
    // which it walks by the layer strides.  The index build then runs as
    // 256-thread blocks, at most two per SM, to leave the store room.
    if (step_mode() == StepMode::kPdl && s.num_tokens == ix.batch && ix.batch <= kStepSelfSlotsBatch) {
      sp.p.self = SelfSlots{ix.prior_len, ix.new_len, ix.page_table, ix.table_index, ix.page_table_stride,
                            ix.num_pages, ix.batch, ix.page_size, ix.max_pages_per_row, ix.num_table_rows,
                            ix.slot64, ix.by_page};
      const uint64_t store_bytes = 4ull * static_cast<uint64_t>(s.num_layers) *
                                   static_cast<uint64_t>(s.num_tokens) * static_cast<uint64_t>(s.row_bytes);
      ix.beside_store = store_bytes >= (48ull << 20) ? 2 : 1;
    }
    rc = launch_index(ix, stream);
    if (rc != YL_OK) return rc;
    return launch_store(sp, s.row_bytes, s.slot_is_int64 != 0, stream, step_mode() == StepMode::kPdl);
  }

  StepParams p;
  p.ix = ix;
  p.st = sp.p;
  p.num_tokens = static_cast<uint32_t>(s.num_tokens);
  const size_t smem = step_smem(ix.batch);
  const uint64_t rows_per_block = static_cast<uint64_t>(kStepThreads / group) * rows;
  const uint64_t row_blocks = (p.st.total_rows + rows_per_block - 1) / rows_per_block;
  const uint64_t fill = static_cast<uint64_t>(ix.indices_cap) +
                        static_cast<uint64_t>(ix.slots_cap > s.num_tokens ? ix.slots_cap - s.num_tokens : 0);
  const uint64_t fill_blocks = (fill + 4 * kStepThreads - 1) / (4 * kStepThreads);
  uint64_t want = row_blocks > fill_blocks ? row_blocks : fill_blocks;
  const uint64_t cap = static_cast<uint64_t>(sm_count()) * blocks_per_sm(reinterpret_cast<const void *>(fn), smem);
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  fn<<<static_cast<unsigned>(want), kStepThreads, smem, stream>>>(p);
  return check_launch("yl_kv_step launch");
}
