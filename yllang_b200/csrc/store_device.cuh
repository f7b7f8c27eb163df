// Device side of the K/V row copy of the store kernels (kv_store.cu), which
// the step (kv_step.cu) launches behind its index build.
//
// Rows are enumerated plane-major: row r in [0, 2 * L * N) is token r % N of
// plane r / N, plane = 2 * layer + {0: K, 1: V}.  A group of G lanes copies one
// row as G * VPL vectors of W bytes; a group takes R rows per iteration and
// issues every load of the iteration before it needs any slot, so the K/V
// reads are in flight while slots are read (or computed) and checked.
#pragma once

#include <climits>
#include <cstdint>

#include "common.cuh"

namespace ylk {

// Step only, decode batches: what the store needs to compute a token's slot
// itself (batch = 0: read the slots the index build writes).
struct SelfSlots {
  const int32_t *prior_len;
  const int32_t *new_len;
  const int32_t *page_table;
  const int32_t *table_index;
  int64_t page_table_stride;
  int64_t num_pages;
  int32_t batch;
  int32_t page_size;
  int32_t max_pages_per_row;
  int32_t num_table_rows;
  int32_t slot64;
  FastDiv by_page;
};

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
  SelfSlots self;
  uint64_t wait_limit_ns;  // bulk-copy kernels: bound of the first wait for a round's rows
};

// ---------------------------------------------------------------------------
// Vector types and cache-hinted global accesses.  The step's input rows are
// read exactly once: non-coherent path, no L1 allocation.
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

// True (on every thread of the block) when every sequence of the batch adds
// exactly one token, so token t is sequence t's new token and the store can
// compute slots itself.  Each thread reads its share of new_len, eight loads
// in flight at a time.
__device__ __forceinline__ bool decode_batch(const SelfSlots &s) {
  int ok = s.batch > 0;
  for (int base = threadIdx.x; base < s.batch; base += 8 * blockDim.x) {
    int32_t v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * static_cast<int>(blockDim.x);
      v[u] = i < s.batch ? __ldg(s.new_len + i) : 1;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) ok &= v[u] == 1;
  }
  return __syncthreads_and(ok) != 0;
}

// Slot of token t of a decode batch, by the index build's rules (slot_at
// over the facts of seq_facts): the prior length clamped at 0; a table row
// outside the table, or a page past the sequence's pages (its row capped at
// max_pages_per_row), gives -1 with no bit (the index build reports those);
// a page id outside the pool, or an int32 slot above INT_MAX, gives -1 and
// sets YL_DEVERR_PAGE_RANGE.
__device__ __forceinline__ int64_t decode_slot(const SelfSlots &s, uint32_t t, uint32_t *error_word) {
  const int32_t pos = max(__ldg(s.prior_len + t), 0);
  const int32_t row = s.table_index ? __ldg(s.table_index + t) : static_cast<int32_t>(t);
  if (s.table_index && (row < 0 || row >= s.num_table_rows)) return -1;
  const int64_t pages = min((static_cast<int64_t>(pos) + s.page_size) / s.page_size,
                            static_cast<int64_t>(s.max_pages_per_row));  // ceil((pos + 1) / ps), capped
  const uint32_t pidx = s.by_page.div(static_cast<uint32_t>(pos));
  if (static_cast<int64_t>(pidx) >= pages) return -1;
  const int32_t page = __ldg(s.page_table + static_cast<int64_t>(row) * s.page_table_stride + pidx);
  const bool in_range = page >= 0 && (s.num_pages <= 0 || page < s.num_pages);
  const int64_t slot = static_cast<int64_t>(page) * s.page_size + (pos - static_cast<int64_t>(pidx) * s.page_size);
  if (in_range && (s.slot64 || slot <= INT_MAX)) return slot;
  raise_deverr(error_word, YL_DEVERR_PAGE_RANGE);
  return -1;
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

// R rows of one lane group held in registers between their loads and stores.
template <int W, int G, int VPL, int R>
struct RowBatch {
  Vec<W> data[R][VPL];
  char *dst[R];
  uint32_t token[R];
  bool live[R];

  // Issue the loads of rows [base, base + R) (those below total_rows).
  __device__ __forceinline__ void load(const StoreParams &p, uint32_t base, uint32_t lane) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint32_t row = base + r;
      live[r] = row < p.total_rows;
      if (live[r]) {
        const RowAddr a = row_addr(p, row, token[r]);
        dst[r] = a.dst_base;
#pragma unroll
        for (int j = 0; j < VPL; ++j) load_vec(data[r][j], a.src + (j * G + lane) * W);
      }
    }
  }

  // Issue the loads of the rows rows[r] for which ok[r] holds.
  __device__ __forceinline__ void load_list(const StoreParams &p, const uint32_t (&rows)[R], const bool (&ok)[R],
                                            uint32_t lane) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      live[r] = ok[r];
      if (live[r]) {
        const RowAddr a = row_addr(p, rows[r], token[r]);
        dst[r] = a.dst_base;
#pragma unroll
        for (int j = 0; j < VPL; ++j) load_vec(data[r][j], a.src + (j * G + lane) * W);
      }
    }
  }

  // Attach row r's slot (skipping it when the slot is not a pool row).
  __device__ __forceinline__ void resolve(const StoreParams &p, int r, int64_t slot) {
    if (live[r]) {
      live[r] = slot_ok(slot, p);
      dst[r] += slot * p.cache_row_stride;
    }
  }

  __device__ __forceinline__ void store(uint32_t lane) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (live[r]) {
#pragma unroll
        for (int j = 0; j < VPL; ++j) store_vec(dst[r] + (j * G + lane) * W, data[r][j]);
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Host-side choice of the fast row shape for a row size and vector width.
// ---------------------------------------------------------------------------
template <int W_, int G_, int VPL_, int R_>
struct RowShape {
  static constexpr int W = W_;      // bytes per vector
  static constexpr int G = G_;      // lanes per row
  static constexpr int VPL = VPL_;  // vectors per lane per row
  static constexpr int R = R_;      // rows per lane group per iteration
};

// Calls f(RowShape<...>{}) with the fast shape for row_bytes at vector width
// w (16 or 32 bytes); returns false when there is none (generic path).
template <typename F>
inline bool dispatch_row_shape(int64_t row_bytes, int w, F &&f) {
  if (w == 16) {
    switch (row_bytes) {
      case 16: f(RowShape<16, 1, 1, 8>{}); return true;
      case 32: f(RowShape<16, 2, 1, 8>{}); return true;
      case 64: f(RowShape<16, 4, 1, 8>{}); return true;
      case 128: f(RowShape<16, 8, 1, 8>{}); return true;
      case 256: f(RowShape<16, 16, 1, 8>{}); return true;
      case 512: f(RowShape<16, 32, 1, 8>{}); return true;
      case 1024: f(RowShape<16, 32, 2, 4>{}); return true;
      case 2048: f(RowShape<16, 32, 4, 2>{}); return true;
      case 4096: f(RowShape<16, 32, 8, 1>{}); return true;
      case 8192: f(RowShape<16, 32, 16, 1>{}); return true;
      default: return false;
    }
  }
  switch (row_bytes) {
    case 256: f(RowShape<32, 8, 1, 8>{}); return true;
    case 512: f(RowShape<32, 16, 1, 8>{}); return true;
    case 1024: f(RowShape<32, 32, 1, 4>{}); return true;
    case 2048: f(RowShape<32, 32, 2, 2>{}); return true;
    case 4096: f(RowShape<32, 32, 4, 1>{}); return true;
    case 8192: f(RowShape<32, 32, 8, 1>{}); return true;
    default: return false;
  }
}

// Vector width of the fast path: 32-byte vectors (ld/st .v8.b32, sm_100) when
// every address and stride is 32-byte aligned, else 16-byte vectors;
// YL_STORE_VECTOR_BYTES=16 forces 16-byte vectors.
int fast_vector_bytes();

// Host halves of the entry points (kv_store.cu, index_build.cu), shared with
// the step (kv_step.cu).  `prepare_*` validate the arguments and fill
// the kernel parameters; `launch_*` launch the separate kernels.
struct StorePlan {
  StoreParams p;
  int unit;         // widest vector unit every address and stride allows
  uintptr_t bits;   // OR of addresses and strides (alignment of the fast path)
};
int prepare_store(const yl_store_args *a, bool need_slots, StorePlan &plan);
// pdl: launch as the programmatic dependent of the previous kernel in the
// stream (it must not write the K/V rows; the slots are read after it ends).
int launch_store(const StorePlan &plan, int64_t row_bytes, bool slot64, cudaStream_t stream, bool pdl);

}  // namespace ylk
