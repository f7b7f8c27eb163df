// One serving step of the path: the batch index build, then the store of
// every layer's new K/V rows under the slot mapping it produces
// (yl_build_index then yl_kv_store, as two launches that overlap).
//
// The index build is a programmatic dependent of whatever kernel precedes it
// (its blocks are placed while that kernel drains and wait for it before
// reading anything), and the store is a programmatic dependent of the index
// build: it issues its first K/V loads, which depend on nothing the index
// build writes, as soon as the index build's blocks have started.  A store
// that reads the slot mapping then waits for the index build; for a decode
// batch (N == B and, checked by every store CTA, every new_len is 1) token t
// is sequence t's new token, so the store computes its slots itself by the
// index build's rules and runs beside it (store_decode_kernel).
//
// Measured and dropped on B200 (decode, 256 sequences, 32 layers): fusing the
// two into one kernel, register-staged (every block scans the batch while its
// first rows are in flight; 16.9-17.1 us, registers cap it at three CTAs per
// SM) or TMA-staged (one CTA per SM stages its rows in shared memory with
// cp.async.bulk; 17.4 us), against 13.4 us for the overlapped launches.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "index_device.cuh"
#include "store_device.cuh"

namespace ylk {

// YL_STEP_MODE=serial runs the two launches without the overlap (the store
// waits for the whole index build and reads its slot mapping), for timing
// the overlap against it; read once per process.
static bool serial_step() {
  static const bool s = [] {
    const char *e = std::getenv("YL_STEP_MODE");
    return e != nullptr && std::strcmp(e, "serial") == 0;
  }();
  return s;
}

// Decode batches up to kStepSelfSlotsBatch sequences have the store compute
// their slots (store_decode_kernel: one slot per lane group and token).
constexpr int kStepSelfSlotsBatch = 16384;

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

  const bool overlap = !serial_step();
  // A decode batch: the store computes its own slots beside the index build,
  // which then runs as 256-thread blocks, at most two per SM (one beside a
  // store of 48 MB or more, whose length hides the index build's latency).
  if (overlap && s.num_tokens == ix.batch && ix.batch <= kStepSelfSlotsBatch) {
    sp.p.self = SelfSlots{ix.prior_len, ix.new_len, ix.page_table, ix.table_index, ix.page_table_stride,
                          ix.num_pages, ix.batch, ix.page_size, ix.max_pages_per_row, ix.num_table_rows,
                          ix.slot64, ix.by_page};
    const uint64_t store_bytes = 4ull * static_cast<uint64_t>(s.num_layers) * static_cast<uint64_t>(s.num_tokens) *
                                 static_cast<uint64_t>(s.row_bytes);
    ix.beside_store = store_bytes >= (48ull << 20) ? 2 : 1;
  }
  rc = launch_index(ix, stream);
  if (rc != YL_OK) return rc;
  return launch_store(sp, s.row_bytes, s.slot_is_int64 != 0, stream, overlap);
}
