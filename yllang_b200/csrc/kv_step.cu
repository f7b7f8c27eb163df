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

#include "common.cuh"
#include "index_device.cuh"
#include "store_device.cuh"

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
  int64_t *scratch = smem;                                // 64 x int64
  int32_t *kvp = reinterpret_cast<int32_t *>(smem + 64);  // [B+1]
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

static size_t step_smem(int batch) { return 64 * sizeof(int64_t) + 2 * (batch + 1) * sizeof(int32_t); }

// How yl_kv_step runs: the index build and a PDL-dependent store (default),
// the one-launch fused kernel (YL_STEP_MODE=fused), or the two launches
// serialised (YL_STEP_MODE=serial).
enum class StepMode { kPdl, kFused, kSerial };
static StepMode step_mode() {
  static const StepMode m = [] {
    const char *e = std::getenv("YL_STEP_MODE");
    if (e != nullptr && std::strcmp(e, "fused") == 0) return StepMode::kFused;
    if (e != nullptr && std::strcmp(e, "serial") == 0) return StepMode::kSerial;
    return StepMode::kPdl;
  }();
  return m;
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
  if (fused) {
    bool found = false;
    if (w == 32 && (sp.bits & 31u) == 0) found = dispatch_row_shape(s.row_bytes, 32, pick);
    if (!found) found = dispatch_row_shape(s.row_bytes, 16, pick);
    fused = found;
  }
  if (!fused || step_mode() != StepMode::kFused) {
    // Two launches: the index build, then the store reading its slot mapping.
    // In PDL mode the store is the index kernel's programmatic dependent: its
    // K/V loads overlap the index build and only the slot reads wait for it.
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
