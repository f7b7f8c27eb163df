// Device side of the batch index build (index_build.cu; the step's decode
// store, store_device.cuh, follows the same slot rules).
//
// The per-sequence page and token counts are exclusive-scanned into
// kv_indptr / qo_indptr offsets (in shared memory, or in the outputs for very
// large batches); every other output element then finds its sequence by a
// binary search over those offsets and gathers from that sequence's
// page-table row.
#pragma once

#include <climits>
#include <cstdint>

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
  int64_t expected_tokens;  // step only: the store's N, checked against the sum of new_len (-1: no check)
  int32_t beside_store;     // step only: the store may run beside this kernel (1), a long one (2); leave it room
};

// int64 words of shared scratch the scan needs: 2 x 32 warp totals, 2 block
// totals, and one word whose low half holds the batch's largest page count.
constexpr int kScanScratch = 67;
constexpr int kScanMaxWord = 66;

// Largest page count of any sequence, after scan_batch.
__device__ __forceinline__ int32_t scanned_max_pages(const int64_t *scratch) {
  return reinterpret_cast<const int32_t *>(scratch)[2 * kScanMaxWord];
}

struct SeqFacts {
  int32_t prior;  // clamped to >= 0
  int32_t fresh;  // new tokens, clamped to >= 0
  int32_t pages;  // np_i after validation and clamping
  int32_t row;    // page-table row
};

// Validated per-sequence facts from the sequence's loaded prior length, new
// length and table row.  Only `report` threads raise error bits so a bad
// input is not reported once per block.
__device__ __forceinline__ SeqFacts facts_of(const IndexParams &p, int32_t pl, int32_t nl, int32_t row, bool report) {
  SeqFacts f;
  if (pl < 0 || nl < 0) {
    if (report) raise_deverr(p.error_word, YL_DEVERR_NEGATIVE_LEN);
    pl = max(pl, 0);
    nl = max(nl, 0);
  }
  f.prior = pl;
  f.fresh = nl;
  f.row = row;
  bool row_ok = true;
  if (p.table_index != nullptr && (row < 0 || row >= p.num_table_rows)) {
    if (report) raise_deverr(p.error_word, YL_DEVERR_TABLE_ROW);
    row_ok = false;
  }
  const int64_t total = static_cast<int64_t>(pl) + nl;
  int64_t np = 0;
  if (row_ok) {
    const int64_t up = total + p.page_size - 1;
    np = up < (1ll << 31) ? static_cast<int64_t>(p.by_page.div(static_cast<uint32_t>(up))) : up / p.page_size;
  }
  if (np > p.max_pages_per_row) {
    if (report) raise_deverr(p.error_word, YL_DEVERR_ROW_OVERFLOW);
    np = p.max_pages_per_row;
  }
  f.pages = static_cast<int32_t>(np);
  return f;
}

__device__ __forceinline__ SeqFacts seq_facts(const IndexParams &p, int i, bool report) {
  return facts_of(p, p.prior_len[i], p.new_len[i], p.table_index != nullptr ? p.table_index[i] : i, report);
}

// Sequences staged per thread per round of the scan (their loads in flight together).
constexpr int kStageUnroll = 8;

// Phase A: page and token counts of all sequences, exclusive-scanned into
// kvp[0..B] and qop[0..B] (shared or global memory).  Thread k owns the
// consecutive sequences [k m, k m + m), m = ceil(B / threads): it loads their
// lengths kStageUnroll at a time (the loads in flight together), writes their
// counts and keeps their sums; then one warp scan of the thread sums, one
// scan of the warp sums, and a second pass over its own sequences turns the
// counts into offsets.  A block scans B sequences with one shuffle scan per
// warp whatever B is (a scan 32 entries at a time costs a shuffle scan per 32
// sequences, which at a few thousand sequences dominated the kernel).
// Returns false (uniformly across the block) when a total passes INT32_MAX;
// the fill must then be skipped.  The batch's largest page count is left in
// scratch for the fill's choice (scanned_max_pages).
template <bool kBig = false>
__device__ inline bool scan_batch(const IndexParams &p, int32_t *kvp, int32_t *qop, int64_t *scratch, bool report) {
  const int B = p.batch;
  const int m = (B + static_cast<int>(blockDim.x) - 1) / static_cast<int>(blockDim.x);
  const int s0 = min(B, static_cast<int>(threadIdx.x) * m), s1 = min(B, s0 + m);
  int32_t *max_word = reinterpret_cast<int32_t *>(scratch) + 2 * kScanMaxWord;
  if (threadIdx.x == 0) *max_word = 0;
  int64_t sa = 0, sb = 0;
  int32_t max_pages = 0;
  for (int base = s0; base < s1; base += kStageUnroll) {
    int32_t pl[kStageUnroll], nl[kStageUnroll], rw[kStageUnroll];
#pragma unroll
    for (int u = 0; u < kStageUnroll; ++u) {
      const int i = base + u;
      if (i < s1) {
        pl[u] = __ldg(p.prior_len + i);
        nl[u] = __ldg(p.new_len + i);
        rw[u] = p.table_index != nullptr ? __ldg(p.table_index + i) : i;
      }
    }
#pragma unroll
    for (int u = 0; u < kStageUnroll; ++u) {
      const int i = base + u;
      if (i < s1) {
        const SeqFacts f = facts_of(p, pl[u], nl[u], rw[u], report);
        kvp[i] = f.pages;
        qop[i] = f.fresh;
        sa += f.pages;
        sb += f.fresh;
        max_pages = max(max_pages, f.pages);
      }
    }
  }
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  int64_t a = sa, b = sb;  // inclusive scan of the thread sums within the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t ua = __shfl_up_sync(0xffffffffu, a, o);
    const int64_t ub = __shfl_up_sync(0xffffffffu, b, o);
    if (lane >= o) {
      a += ua;
      b += ub;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) max_pages = max(max_pages, __shfl_xor_sync(0xffffffffu, max_pages, o));
  if (lane == 31) {
    scratch[warp] = a;
    scratch[32 + warp] = b;
  }
  __syncthreads();  // warp sums, and the max word's reset, visible
  if (lane == 0) atomicMax(max_word, max_pages);
  if (warp == 0) {
    int64_t wa = lane < nwarps ? scratch[lane] : 0, wb = lane < nwarps ? scratch[32 + lane] : 0;
    const int64_t wa0 = wa, wb0 = wb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t ua = __shfl_up_sync(0xffffffffu, wa, o);
      const int64_t ub = __shfl_up_sync(0xffffffffu, wb, o);
      if (lane >= o) {
        wa += ua;
        wb += ub;
      }
    }
    if (lane < nwarps) {
      scratch[lane] = wa - wa0;  // exclusive warp offsets
      scratch[32 + lane] = wb - wb0;
    }
    if (lane == 31) {
      scratch[64] = wa;  // block totals
      scratch[65] = wb;
    }
  }
  __syncthreads();
  const int64_t ta = scratch[64], tb = scratch[65];
  if (ta > INT_MAX || tb > INT_MAX) {
    if (report && threadIdx.x == 0) raise_deverr(p.error_word, YL_DEVERR_INDPTR_OVERFLOW);
    return false;
  }
  // every prefix is at most its total, so the offsets fit in int32
  int32_t oa = static_cast<int32_t>(scratch[warp] + a - sa), ob = static_cast<int32_t>(scratch[32 + warp] + b - sb);
  for (int i = s0; i < s1; ++i) {
    const int32_t ca = kvp[i], cb = qop[i];
    kvp[i] = oa;
    qop[i] = ob;
    oa += ca;
    ob += cb;
  }
  if (threadIdx.x == 0) {
    kvp[B] = static_cast<int32_t>(ta);
    qop[B] = static_cast<int32_t>(tb);
  }
  __syncthreads();
  return true;
}

// Largest i in [0, n] with off[i] <= e, given off[0] <= e < off[n], by a
// branchless walk down a power-of-two ladder (`top` = the largest power of
// two <= n, or 0 when n == 0); 32-bit, for the fill loops.
__device__ __forceinline__ int find_seq32(const int32_t *off, int n, int32_t e, int top) {
  int lo = 0;
  for (int step = top; step > 0; step >>= 1) {
    const int c = lo + step;
    if (c <= n && off[c] <= e) lo = c;
  }
  return lo;
}

__device__ __forceinline__ int pow2_floor(int n) { return n > 0 ? 1 << (31 - __clz(n)) : 0; }

__device__ __forceinline__ void write_slot(const IndexParams &p, int64_t t, int64_t slot) {
  if (p.slot64) static_cast<int64_t *>(p.slot_mapping)[t] = slot;
  else static_cast<int32_t *>(p.slot_mapping)[t] = static_cast<int32_t>(slot);
}

// Slot of position `pos` of sequence i, or -1 when it has none (the position
// is past the sequence's page-table row, or its page is not a pool page).
__device__ __forceinline__ int64_t slot_at(const IndexParams &p, const int32_t *kvp, int i, int64_t pos) {
  const int32_t pages = kvp[i + 1] - kvp[i];
  if (pos < 0 || pos >= (1ll << 31)) return -1;
  const uint32_t pidx = p.by_page.div(static_cast<uint32_t>(pos));
  if (static_cast<int64_t>(pidx) >= pages) return -1;
  const int32_t row = p.table_index ? __ldg(p.table_index + i) : i;
  const int32_t page = __ldg(p.page_table + static_cast<int64_t>(row) * p.page_table_stride + pidx);
  const bool in_range = page >= 0 && (p.num_pages <= 0 || page < p.num_pages);
  const int64_t s = static_cast<int64_t>(page) * p.page_size + (pos - static_cast<int64_t>(pidx) * p.page_size);
  if (in_range && (p.slot64 || s <= INT_MAX)) return s;
  raise_deverr(p.error_word, YL_DEVERR_PAGE_RANGE);
  return -1;
}

// Phase C for the elements [begin, end) of [kv_indices | slot_mapping]: one
// element per thread per pass (U per pass for big batches), its sequence
// found by a branchless search over
// the scanned offsets, gathered from that sequence's page-table row
// (coalesced row reads and output writes).  The whole fill space is below
// 2^31 elements (checked on the host), so element arithmetic is 32-bit.
// Slot entries past qo_indptr[B] (up to the slot capacity) are written as -1.
// Each element belongs to exactly one block, so every block reports its own.
// Measured on B200 and slower for the decode batch (under one element per
// thread): warp-cooperative searches (two per chunk, then a per-lane search
// of the chunk's span), multi-element unrolled passes, and per-block walks
// over the spanned sequences (latency-bound at one element per thread; any
// serial per-block search lands on its critical path).
template <int U>
__device__ inline void fill_range(const IndexParams &p, const int32_t *kvp, const int32_t *qop, int32_t n_idx,
                                  int32_t begin, int32_t end) {
  const int32_t n_tok = qop[p.batch];
  const int top = pow2_floor(p.batch);
  const int32_t kv_end = min(end, n_idx);
  const int32_t step = static_cast<int32_t>(blockDim.x);
  // U elements per thread per pass: every search, then every page-table load,
  // then every store, so a thread with several elements has them in flight
  // together (the big-batch kernel; U = 1 elsewhere).
  for (int32_t e0 = begin + static_cast<int32_t>(threadIdx.x); e0 < kv_end; e0 += U * step) {
    int seq[U];
    int32_t page[U];
    // one search for the first element; a later element in the same
    // sequence (long rows: page size 1, long contexts) needs one shared-memory
    // load instead of its own search, and the other searches stay independent
    const int s0 = e0 < kv_end ? find_seq32(kvp, p.batch, e0, top) : -1;
    const int32_t s0_end = s0 >= 0 ? kvp[s0 + 1] : 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int32_t e = e0 + u * step;
      seq[u] = e >= kv_end ? -1 : (e < s0_end ? s0 : find_seq32(kvp, p.batch, e, top));
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (seq[u] >= 0) {
        const int32_t row = p.table_index ? __ldg(p.table_index + seq[u]) : seq[u];
        page[u] = __ldg(p.page_table + static_cast<int64_t>(row) * p.page_table_stride + (e0 + u * step - kvp[seq[u]]));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (seq[u] >= 0) {
        if (p.num_pages > 0 && (page[u] < 0 || page[u] >= p.num_pages)) raise_deverr(p.error_word, YL_DEVERR_PAGE_RANGE);
        p.kv_indices[e0 + u * step] = page[u];
      }
    }
  }
  for (int32_t e = max(begin, n_idx) + static_cast<int32_t>(threadIdx.x); e < end; e += step) {
    const int32_t t = e - n_idx;
    int64_t slot = -1;
    if (t < n_tok) {
      const int i = find_seq32(qop, p.batch, t, top);
      slot = slot_at(p, kvp, i, static_cast<int64_t>(max(__ldg(p.prior_len + i), 0)) + (t - qop[i]));
    }
    write_slot(p, t, slot);
  }
}

// kv_indices by sequence: each sequence's page-table row is copied by wps
// warps of the grid (wps = warps in the grid / B, 1 to 8; warp part q of a
// sequence takes its pages q*32 + lane + 32*wps*k), kSeqCopyUnroll pages per
// lane in flight; no search.  For batches with more pages than threads,
// where the per-element search's instructions dominate.  Eight pages per lane
// (four before) took one rank's decode step at 2,048 sequences from 21.5 to
// 20.4 us and Qwen2-72B decode at one head per GPU from 14.0 to 13.7 us;
// sixteen lost on the latter (16.1 us).
constexpr int kSeqCopyUnroll = 8;
__device__ inline void fill_kv_by_sequence(const IndexParams &p, const int32_t *kvp, int32_t n_idx) {
  const int lane = threadIdx.x & 31;
  const int warps = static_cast<int>((gridDim.x * blockDim.x) >> 5);
  const int wps = max(1, min(8, warps / max(p.batch, 1)));
  const int gw = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int part = gw % wps;
  const int stride = 32 * wps;
  for (int i = gw / wps; i < p.batch; i += warps / wps) {
    const int32_t off = kvp[i];
    const int32_t n = min(kvp[i + 1], n_idx) - off;  // the capacity clamps the tail
    if (n <= 0) continue;
    const int32_t row = p.table_index ? __ldg(p.table_index + i) : i;
    const int32_t *src = p.page_table + static_cast<int64_t>(row) * p.page_table_stride;
    int32_t *dst = p.kv_indices + off;
    for (int32_t j0 = part * 32 + lane; j0 < n; j0 += stride * kSeqCopyUnroll) {
      int32_t page[kSeqCopyUnroll];
#pragma unroll
      for (int u = 0; u < kSeqCopyUnroll; ++u)
        if (j0 + stride * u < n) page[u] = __ldg(src + j0 + stride * u);
#pragma unroll
      for (int u = 0; u < kSeqCopyUnroll; ++u) {
        if (j0 + stride * u < n) {
          if (p.num_pages > 0 && (page[u] < 0 || page[u] >= p.num_pages)) raise_deverr(p.error_word, YL_DEVERR_PAGE_RANGE);
          dst[j0 + stride * u] = page[u];
        }
      }
    }
  }
}

// Slots of tokens [0, slot capacity), grid-strided over threads (entries past
// qo_indptr[B] are -1).
__device__ inline void fill_slots_strided(const IndexParams &p, const int32_t *kvp, const int32_t *qop) {
  const int32_t n_tok = qop[p.batch];
  const int top = pow2_floor(p.batch);
  const int64_t n_slot = p.slot_mapping ? p.slots_cap : 0;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n_slot;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t slot = -1;
    if (t < n_tok) {
      const int i = find_seq32(qop, p.batch, static_cast<int32_t>(t), top);
      slot = slot_at(p, kvp, i, static_cast<int64_t>(max(__ldg(p.prior_len + i), 0)) + (t - qop[i]));
    }
    write_slot(p, t, slot);
  }
}

// True when the sequence-warp fill suits the batch: more pages than threads
// in the grid (else one element per thread is already a single pass), at
// least 32 pages per sequence on average (a warp's lanes busy) and no
// sequence above 2,048 pages (no warp left copying long after the others).
__device__ __forceinline__ bool fill_by_sequence_suits(const IndexParams &p, const int32_t *kvp, int32_t max_pages) {
  return p.batch > 0 && kvp[p.batch] > static_cast<int64_t>(gridDim.x) * blockDim.x &&
         kvp[p.batch] >= 32ll * p.batch && max_pages <= 2048;
}

// Phase B: per-sequence outputs for i in [first, B], stepping by `step`.
__device__ inline void write_seq_outputs(const IndexParams &p, const int32_t *kvp, const int32_t *qop, int64_t first,
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

// Split of the fill space [kv_indices | slot_mapping] among blocks, with the
// capacity and token-count checks.
template <int U>
__device__ __forceinline__ void fill_block_share(const IndexParams &p, const int32_t *kvp, const int32_t *qop,
                                                 bool report, bool by_sequence = false) {
  if (report && threadIdx.x == 0 && p.expected_tokens >= 0 && qop[p.batch] != p.expected_tokens)
    raise_deverr(p.error_word, YL_DEVERR_TOKEN_COUNT);
  int64_t n_idx = p.kv_indices ? kvp[p.batch] : 0;
  const int64_t n_slot = p.slot_mapping ? p.slots_cap : 0;
  if (n_idx > p.indices_cap) {
    if (report && threadIdx.x == 0) raise_deverr(p.error_word, YL_DEVERR_INDICES_CAP);
    n_idx = p.indices_cap;
  }
  if (p.slot_mapping && qop[p.batch] > p.slots_cap && report && threadIdx.x == 0)
    raise_deverr(p.error_word, YL_DEVERR_SLOTS_CAP);
  if (by_sequence) {
    fill_kv_by_sequence(p, kvp, static_cast<int32_t>(n_idx));
    fill_slots_strided(p, kvp, qop);
    return;
  }
  const int64_t work = n_idx + n_slot;  // < 2^31 (checked on the host)
  const int64_t chunk = (work + gridDim.x - 1) / gridDim.x;
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * chunk;
  const int64_t end = min(begin + chunk, work);
  if (begin < end)
    fill_range<U>(p, kvp, qop, static_cast<int32_t>(n_idx), static_cast<int32_t>(begin), static_cast<int32_t>(end));
}

// Host halves of yl_build_index (index_build.cu), shared with the step:
// prepare_index validates the arguments and fills the kernel parameters,
// launch_index launches the index kernels.
int prepare_index(const yl_index_args *a, IndexParams &p);
int launch_index(const IndexParams &p, cudaStream_t stream);

}  // namespace ylk
