// Batch index build for sm_100a: from per-sequence lengths and page-table rows
// produce kv_indptr / kv_indices / kv_last_page_len / qo_indptr / slot_mapping.
//
// The reference builds its per-step indices on the host, one libtorch scalar
// op per element (Make2DIndices, src/include/batch/batch_manager.h:30-51,
// called from NextBatch, batch_manager.h:97-112), for page size 1.  Here the
// whole batch is one launch:
//
//   phase A  every block redundantly computes each sequence's page count and
//            new-token count and exclusive-scans both into shared memory
//            (B <= kSmemBatchLimit; the batch is a few KB, an L2 hit for every
//            block after the first, so this avoids any inter-block handshake);
//   phase B  the blocks write kv_indptr, qo_indptr and kv_last_page_len;
//   phase C  the concatenated element space [kv_indices | slot_mapping] is cut
//            into equal contiguous chunks, one per block; each thread finds its
//            element's sequence by binary search over the scanned offsets and
//            gathers from that sequence's page-table row, so reads of a row and
//            writes of kv_indices are both coalesced.
//
// Batches above kSmemBatchLimit take a two-launch form: one block scans into
// the kv_indptr / qo_indptr outputs, then the fill reads them from global
// memory.  Neither form needs memory beyond the caller's outputs.
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace ylk {

struct IndexParams {
  const int32_t *prior_len;
  const int32_t *new_len;
  const int32_t *page_table;
  const int32_t *table_index;
  int64_t page_table_stride;
  int64_t num_pages;
  int64_t indices_cap;
  int64_t slots_cap;
  int32_t *kv_indptr;
  int32_t *kv_indices;
  int32_t *last_page_len;
  int32_t *qo_indptr;
  void *slot_mapping;
  uint32_t *error_word;
  int32_t num_table_rows;
  int32_t max_pages_per_row;
  int32_t page_size;
  int32_t batch;
  int32_t slot64;
  FastDiv by_page;
};

constexpr int kIndexThreads = 1024;
constexpr int kSmemBatchLimit = 16384;

struct SeqFacts {
  int32_t prior;  // clamped to >= 0
  int32_t fresh;  // new tokens, clamped to >= 0
  int32_t pages;  // np_i after validation and clamping
  int32_t row;    // page-table row
};

// Validated per-sequence facts.  Only `report` threads raise error bits so a
// bad input is not reported once per block.
__device__ __forceinline__ SeqFacts seq_facts(const IndexParams &p, int i, bool report) {
  SeqFacts f;
  int32_t pl = p.prior_len[i];
  int32_t nl = p.new_len[i];
  if (pl < 0 || nl < 0) {
    if (report) raise_deverr(p.error_word, YL_DEVERR_NEGATIVE_LEN);
    pl = max(pl, 0);
    nl = max(nl, 0);
  }
  f.prior = pl;
  f.fresh = nl;
  f.row = i;
  bool row_ok = true;
  if (p.table_index != nullptr) {
    f.row = p.table_index[i];
    if (f.row < 0 || f.row >= p.num_table_rows) {
      if (report) raise_deverr(p.error_word, YL_DEVERR_TABLE_ROW);
      row_ok = false;
    }
  }
  const int64_t total = static_cast<int64_t>(pl) + nl;
  int64_t np = row_ok ? (total + p.page_size - 1) / p.page_size : 0;
  if (np > p.max_pages_per_row) {
    if (report) raise_deverr(p.error_word, YL_DEVERR_ROW_OVERFLOW);
    np = p.max_pages_per_row;
  }
  f.pages = static_cast<int32_t>(np);
  return f;
}

// Exclusive block scan of two int64 values per thread.  `scratch` holds 64
// int64; returns the block totals through ta/tb.  Ends synchronised.
__device__ __forceinline__ void block_scan2(int64_t &a, int64_t &b, int64_t &ta, int64_t &tb, int64_t *scratch) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int64_t a0 = a, b0 = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t xa = __shfl_up_sync(0xffffffffu, a, o);
    const int64_t xb = __shfl_up_sync(0xffffffffu, b, o);
    if (lane >= o) {
      a += xa;
      b += xb;
    }
  }
  if (lane == 31) {
    scratch[warp] = a;
    scratch[32 + warp] = b;
  }
  __syncthreads();
  if (warp == 0) {
    int64_t x = lane < nwarps ? scratch[lane] : 0;
    int64_t y = lane < nwarps ? scratch[32 + lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t xx = __shfl_up_sync(0xffffffffu, x, o);
      const int64_t yy = __shfl_up_sync(0xffffffffu, y, o);
      if (lane >= o) {
        x += xx;
        y += yy;
      }
    }
    scratch[lane] = x;
    scratch[32 + lane] = y;
  }
  __syncthreads();
  const int64_t pa = warp > 0 ? scratch[warp - 1] : 0;
  const int64_t pb = warp > 0 ? scratch[32 + warp - 1] : 0;
  ta = scratch[nwarps - 1];
  tb = scratch[32 + nwarps - 1];
  a = pa + a - a0;
  b = pb + b - b0;
  __syncthreads();
}

// Phase A: scan page and token counts of all sequences into kvp[0..B] and
// qop[0..B] (shared or global memory).  Returns false when a sum passes
// INT32_MAX; the fill must then be skipped.
__device__ bool scan_batch(const IndexParams &p, int32_t *kvp, int32_t *qop, int64_t *scratch, bool report) {
  int64_t carry_kv = 0, carry_qo = 0;
  for (int tile = 0; tile < p.batch; tile += blockDim.x) {
    const int i = tile + threadIdx.x;
    int64_t a = 0, b = 0;
    if (i < p.batch) {
      const SeqFacts f = seq_facts(p, i, report);
      a = f.pages;
      b = f.fresh;
    }
    int64_t ta, tb;
    block_scan2(a, b, ta, tb, scratch);
    if (i < p.batch) {
      kvp[i] = static_cast<int32_t>(carry_kv + a);
      qop[i] = static_cast<int32_t>(carry_qo + b);
    }
    carry_kv += ta;
    carry_qo += tb;
    if (carry_kv > INT_MAX || carry_qo > INT_MAX) {
      if (report && threadIdx.x == 0) raise_deverr(p.error_word, YL_DEVERR_INDPTR_OVERFLOW);
      return false;
    }
  }
  if (threadIdx.x == 0) {
    kvp[p.batch] = static_cast<int32_t>(carry_kv);
    qop[p.batch] = static_cast<int32_t>(carry_qo);
  }
  __syncthreads();
  return true;
}

// Largest i in [0, n) with off[i] <= e, given off[0] <= e < off[n].
__device__ __forceinline__ int find_seq(const int32_t *off, int n, int64_t e) {
  int lo = 0, hi = n;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (off[mid] <= e) lo = mid; else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ void write_slot(const IndexParams &p, int64_t t, int64_t slot) {
  if (p.slot64) static_cast<int64_t *>(p.slot_mapping)[t] = slot;
  else static_cast<int32_t *>(p.slot_mapping)[t] = static_cast<int32_t>(slot);
}

// Phase C for the elements [begin, end) of [kv_indices | slot_mapping].  Each
// element belongs to exactly one block, so every block reports its own.
__device__ void fill_range(const IndexParams &p, const int32_t *kvp, const int32_t *qop, int64_t n_idx,
                           int64_t begin, int64_t end) {
  const int64_t ps = p.page_size;
  for (int64_t e = begin + threadIdx.x; e < end; e += blockDim.x) {
    if (e < n_idx) {
      const int i = find_seq(kvp, p.batch, e);
      const int64_t col = e - kvp[i];
      const int32_t row = p.table_index ? p.table_index[i] : i;
      const int32_t page = p.page_table[static_cast<int64_t>(row) * p.page_table_stride + col];
      if (p.num_pages > 0 && (page < 0 || page >= p.num_pages))
        raise_deverr(p.error_word, YL_DEVERR_PAGE_RANGE);
      p.kv_indices[e] = page;
    } else {
      const int64_t t = e - n_idx;
      const int i = find_seq(qop, p.batch, t);
      const int64_t pos = static_cast<int64_t>(max(p.prior_len[i], 0)) + (t - qop[i]);
      const int32_t pages = kvp[i + 1] - kvp[i];
      int64_t slot = -1;
      if (pos < (1ll << 31)) {
        const uint32_t pidx = p.by_page.div(static_cast<uint32_t>(pos));
        if (static_cast<int64_t>(pidx) < pages) {
          const int32_t row = p.table_index ? p.table_index[i] : i;
          const int32_t page = p.page_table[static_cast<int64_t>(row) * p.page_table_stride + pidx];
          const bool in_range = page >= 0 && (p.num_pages <= 0 || page < p.num_pages);
          const int64_t s = static_cast<int64_t>(page) * ps + (pos - static_cast<int64_t>(pidx) * ps);
          if (in_range && (p.slot64 || s <= INT_MAX)) slot = s;
          else raise_deverr(p.error_word, YL_DEVERR_PAGE_RANGE);
        }
      }
      write_slot(p, t, slot);
    }
  }
}

// Phase B: per-sequence outputs for i in [first, B], stepping by `step`.
__device__ void write_seq_outputs(const IndexParams &p, const int32_t *kvp, const int32_t *qop, int64_t first,
                                  int64_t step, bool to_global_indptr) {
  for (int64_t i = first; i <= p.batch; i += step) {
    if (to_global_indptr) {
      p.kv_indptr[i] = kvp[i];
      p.qo_indptr[i] = qop[i];
    }
    if (i < p.batch && p.last_page_len != nullptr) {
      const int32_t pages = kvp[i + 1] - kvp[i];
      const int64_t total = static_cast<int64_t>(max(p.prior_len[i], 0)) + max(p.new_len[i], 0);
      p.last_page_len[i] = pages == 0 ? 0 : static_cast<int32_t>((total - 1) % p.page_size + 1);
    }
  }
}

// Split of the fill space among blocks, with the capacity checks.
__device__ __forceinline__ void fill_block_share(const IndexParams &p, const int32_t *kvp, const int32_t *qop,
                                                 bool report) {
  int64_t n_idx = p.kv_indices ? kvp[p.batch] : 0;
  int64_t n_slot = p.slot_mapping ? qop[p.batch] : 0;
  if (n_idx > p.indices_cap) {
    if (report && threadIdx.x == 0) raise_deverr(p.error_word, YL_DEVERR_INDICES_CAP);
    n_idx = p.indices_cap;
  }
  if (n_slot > p.slots_cap) {
    if (report && threadIdx.x == 0) raise_deverr(p.error_word, YL_DEVERR_SLOTS_CAP);
    n_slot = p.slots_cap;
  }
  const int64_t work = n_idx + n_slot;
  const int64_t chunk = (work + gridDim.x - 1) / gridDim.x;
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * chunk;
  const int64_t end = min(begin + chunk, work);
  if (begin < end) fill_range(p, kvp, qop, n_idx, begin, end);
}

// Single-launch form (B <= kSmemBatchLimit).
__global__ void __launch_bounds__(kIndexThreads) build_index_kernel(const __grid_constant__ IndexParams p) {
  extern __shared__ int64_t smem[];
  int64_t *scratch = smem;                                   // 64 x int64
  int32_t *kvp = reinterpret_cast<int32_t *>(smem + 64);     // [B+1]
  int32_t *qop = kvp + (p.batch + 1);                        // [B+1]
  const bool report = blockIdx.x == 0;
  if (!scan_batch(p, kvp, qop, scratch, report)) return;
  write_seq_outputs(p, kvp, qop, static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x,
                    static_cast<int64_t>(gridDim.x) * blockDim.x, true);
  fill_block_share(p, kvp, qop, report);
}

// Two-launch form, launch 1 (one block): scan straight into the outputs.  On
// overflow kv_indptr[B] is set to -1 so that launch 2 skips the fill.
__global__ void __launch_bounds__(kIndexThreads) scan_index_kernel(const __grid_constant__ IndexParams p) {
  __shared__ int64_t scratch[64];
  if (!scan_batch(p, p.kv_indptr, p.qo_indptr, scratch, true)) {
    if (threadIdx.x == 0) p.kv_indptr[p.batch] = -1;
    return;
  }
  write_seq_outputs(p, p.kv_indptr, p.qo_indptr, threadIdx.x, blockDim.x, false);
}

// Two-launch form, launch 2: fill from the scanned outputs.
__global__ void __launch_bounds__(kIndexThreads) fill_index_kernel(const __grid_constant__ IndexParams p) {
  if (p.kv_indptr[p.batch] < 0) return;
  fill_block_share(p, p.kv_indptr, p.qo_indptr, blockIdx.x == 0);
}

static size_t single_launch_smem(int batch) { return 64 * sizeof(int64_t) + 2 * (batch + 1) * sizeof(int32_t); }

// Opt the single-launch kernel into > 48 KB dynamic shared memory once per device.
static int ensure_smem_attr() {
  static std::mutex mu;
  static std::vector<char> done;
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(done.size()) <= dev) done.resize(dev + 1, 0);
  if (!done[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(build_index_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(single_launch_smem(kSmemBatchLimit)));
    if (e != cudaSuccess) {
      set_last_error(std::string("yl_build_index: cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      return YL_ERR_CUDA;
    }
    done[dev] = 1;
  }
  return YL_OK;
}

}  // namespace ylk

extern "C" int yl_build_index(const yl_index_args *a, cudaStream_t stream) {
  using namespace ylk;
  clear_last_error();
  if (a == nullptr) return fail(YL_ERR_NULL_ARG, "yl_build_index: args is NULL");
  if (a->batch_size < 0) return fail(YL_ERR_BAD_SIZE, "yl_build_index: batch_size=%lld < 0", a->batch_size);
  if (a->page_size < 1) return fail(YL_ERR_BAD_SIZE, "yl_build_index: page_size=%lld < 1", a->page_size);
  if (a->max_pages_per_row < 0)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: max_pages_per_row=%lld < 0", a->max_pages_per_row);
  if (a->kv_indices_capacity < 0 || a->slot_capacity < 0)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: negative capacity (%lld, %lld)", a->kv_indices_capacity,
                a->slot_capacity);
  if (a->slot_is_int64 != 0 && a->slot_is_int64 != 1)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: slot_is_int64=%lld must be 0 or 1", a->slot_is_int64);
  if (!a->kv_indptr || !a->qo_indptr)
    return fail(YL_ERR_NULL_ARG, "yl_build_index: kv_indptr and qo_indptr are required");
  if (a->batch_size > 0 && (!a->prior_len || !a->new_len))
    return fail(YL_ERR_NULL_ARG, "yl_build_index: prior_len and new_len are required");
  const bool wants_gather = (a->kv_indices && a->kv_indices_capacity > 0) || (a->slot_mapping && a->slot_capacity > 0);
  if (a->batch_size > 0 && wants_gather && !a->page_table)
    return fail(YL_ERR_NULL_ARG, "yl_build_index: page_table is required for kv_indices / slot_mapping");
  if (a->table_index && a->num_table_rows <= 0)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: num_table_rows=%lld must be > 0 with table_index",
                a->num_table_rows);
  if (!a->table_index && a->num_table_rows > 0 && a->num_table_rows < a->batch_size)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: %lld page-table rows for a batch of %lld", a->num_table_rows,
                a->batch_size);
  if (a->page_table_stride < 0)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: page_table_stride=%lld < 0", a->page_table_stride);
  if (a->slot_mapping && (reinterpret_cast<uintptr_t>(a->slot_mapping) & (a->slot_is_int64 ? 7u : 3u)))
    return fail(YL_ERR_ALIGNMENT, "yl_build_index: slot_mapping is not aligned to its element size");

  IndexParams p;
  p.prior_len = a->prior_len;
  p.new_len = a->new_len;
  p.page_table = a->page_table;
  p.table_index = a->table_index;
  p.page_table_stride = a->page_table_stride;
  p.num_pages = a->num_pages;
  p.indices_cap = a->kv_indices ? a->kv_indices_capacity : 0;
  p.slots_cap = a->slot_mapping ? a->slot_capacity : 0;
  p.kv_indptr = a->kv_indptr;
  p.kv_indices = a->kv_indices;
  p.last_page_len = a->kv_last_page_len;
  p.qo_indptr = a->qo_indptr;
  p.slot_mapping = a->slot_mapping;
  p.error_word = a->error_word;
  p.num_table_rows = a->num_table_rows;
  p.max_pages_per_row = a->max_pages_per_row;
  p.page_size = a->page_size;
  p.batch = a->batch_size;
  p.slot64 = a->slot_is_int64;
  p.by_page = FastDiv(static_cast<uint32_t>(a->page_size));

  // Blocks: enough for ~2 fill elements per thread, at most one per SM.
  const int64_t work = p.indices_cap + p.slots_cap;
  int64_t blocks = (work + 2 * kIndexThreads - 1) / (2 * kIndexThreads);
  const int64_t sms = sm_count();
  if (blocks < 1) blocks = 1;
  if (blocks > sms) blocks = sms;

  if (a->batch_size <= kSmemBatchLimit) {
    const int rc = ensure_smem_attr();
    if (rc != YL_OK) return rc;
    build_index_kernel<<<static_cast<unsigned>(blocks), kIndexThreads, single_launch_smem(a->batch_size), stream>>>(p);
    return check_launch("yl_build_index launch");
  }
  scan_index_kernel<<<1, kIndexThreads, 0, stream>>>(p);
  int rc = check_launch("yl_build_index scan launch");
  if (rc != YL_OK) return rc;
  fill_index_kernel<<<static_cast<unsigned>(blocks), kIndexThreads, 0, stream>>>(p);
  return check_launch("yl_build_index fill launch");
}
