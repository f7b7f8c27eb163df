// Device page allocator for sm_100a: the free-page list and page table of
// KVCacheManager (src/include/kvcache/cache_manager.h:105-155) on the device.
//
// One CTA of 1024 threads per call.  Pass 1 walks the batch in chunks of
// 1024 sequences (one per thread), checks every input (a row named twice
// included, through a shared-memory bitmap of the rows) and sums the pages the
// call moves with a block scan; the call then either fails as a whole (error
// bits, nothing written) or pass 2 walks the chunks again, recomputing each
// sequence's offset from the running scan, and moves the page ids.  The
// work is a few kilobytes of int32 traffic: the cost is one launch and the
// dependent loads, which is what a single CTA keeps short.
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <cstdio>
#include <string>

#include "common.cuh"

namespace ylk {

constexpr int kPoolThreads = 1024;

struct PoolParams {
  int32_t *free_pages;
  int32_t *free_count;
  int64_t capacity;
  int32_t *table;
  const int32_t *len_a;  // reserve: prior_len; release: num_tokens
  const int32_t *len_b;  // reserve: new_len;   release: unused
  const int32_t *rows;   // reserve: table_index (NULL: row i); release: rows
  int64_t stride;
  int32_t num_rows;
  int32_t max_pages;
  int32_t page_size;
  int32_t n;  // sequences (reserve) or rows to release
  uint32_t *error_word;
};

// Exclusive scan of v over the block (kPoolThreads threads); *total gets the
// block sum on every thread.  Every thread must call it.
__device__ __forceinline__ int64_t block_exclusive_scan(int64_t v, int64_t &total, int64_t *sums) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t w = sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    sums[lane] = w;
  }
  __syncthreads();
  const int64_t before = warp == 0 ? 0 : sums[warp - 1];
  total = sums[31];
  __syncthreads();  // sums is reused by the next call
  return before + x - v;
}

__device__ __forceinline__ int64_t pages_for(int64_t tokens, int32_t page_size) {
  return (tokens + page_size - 1) / page_size;
}

// Reserve, per sequence i: its row, the pages it holds and the pages it lacks.
__device__ __forceinline__ uint32_t reserve_need(const PoolParams &p, int32_t i, int32_t &row, int64_t &held,
                                                 int64_t &lack) {
  const int32_t prior = p.len_a[i], fresh = p.len_b[i];
  row = p.rows != nullptr ? p.rows[i] : i;
  held = lack = 0;
  if (prior < 0 || fresh < 0) return YL_DEVERR_NEGATIVE_LEN;
  if (row < 0 || row >= p.num_rows) return YL_DEVERR_TABLE_ROW;
  held = pages_for(prior, p.page_size);
  const int64_t need = pages_for(static_cast<int64_t>(prior) + fresh, p.page_size);
  if (need > p.max_pages) {
    held = 0;
    return YL_DEVERR_ROW_OVERFLOW;
  }
  lack = need - held;
  return 0;
}

// Release, per row r: the row and the pages it gives back.
__device__ __forceinline__ uint32_t release_count(const PoolParams &p, int32_t r, int32_t &row, int64_t &count) {
  const int32_t tokens = p.len_a[r];
  row = p.rows[r];
  count = 0;
  if (tokens < 0) return YL_DEVERR_NEGATIVE_LEN;
  if (row < 0 || row >= p.num_rows) return YL_DEVERR_TABLE_ROW;
  const int64_t c = pages_for(tokens, p.page_size);
  if (c > p.max_pages) return YL_DEVERR_ROW_OVERFLOW;
  count = c;
  return 0;
}

__device__ __forceinline__ bool page_ok(int32_t id, int64_t capacity) { return id >= 0 && id < capacity; }

// Sets s_err to the OR of every thread's err (all threads call it).
__device__ __forceinline__ uint32_t block_or(uint32_t err, uint32_t *s_err) {
  if (err) atomicOr(s_err, err);
  __syncthreads();
  return *s_err;
}

// Rows of the table marked at once by the duplicate check: a 32 KB bitmap in
// shared memory covers a window of 262,144 consecutive rows.
constexpr int kRowBitmapWords = 8192;
constexpr int64_t kRowWindow = 32ll * kRowBitmapWords;

// YL_DEVERR_DUPLICATE_ROW (on every thread) when one row in
// [0, num_rows) appears twice among rows[0, n): two sequences of a reserve
// would fill one page-table row, or a release would put one row's pages on
// the free list twice.  Rows outside the table are skipped (they carry their
// own bit).  The bitmap walks the windows between the smallest and largest
// row named, so a batch of a few thousand rows takes one window.  All
// threads call it.
__device__ uint32_t duplicate_rows(const int32_t *rows, int32_t n, int32_t num_rows, uint32_t *bits,
                                   int32_t *s_lo, int32_t *s_hi) {
  if (rows == nullptr || n < 2) return 0;
  if (threadIdx.x == 0) {
    *s_lo = INT32_MAX;
    *s_hi = -1;
  }
  __syncthreads();
  int32_t lo = INT32_MAX, hi = -1;
  for (int32_t i = threadIdx.x; i < n; i += kPoolThreads) {
    const int32_t r = rows[i];
    if (r >= 0 && r < num_rows) {
      lo = min(lo, r);
      hi = max(hi, r);
    }
  }
  if (hi >= 0) {
    atomicMin(s_lo, lo);
    atomicMax(s_hi, hi);
  }
  __syncthreads();
  const int64_t first = *s_lo, last = *s_hi;
  uint32_t dup = 0;
  for (int64_t w0 = first; w0 <= last; w0 += kRowWindow) {
    for (int k = threadIdx.x; k < kRowBitmapWords; k += kPoolThreads) bits[k] = 0;
    __syncthreads();
    for (int32_t i = threadIdx.x; i < n; i += kPoolThreads) {
      const int64_t off = static_cast<int64_t>(rows[i]) - w0;
      if (rows[i] < 0 || rows[i] >= num_rows || off < 0 || off >= kRowWindow) continue;
      const uint32_t bit = 1u << (off & 31);
      if (atomicOr(bits + (off >> 5), bit) & bit) dup = YL_DEVERR_DUPLICATE_ROW;
    }
    __syncthreads();  // the next window clears the bitmap
  }
  return __syncthreads_or(dup) ? YL_DEVERR_DUPLICATE_ROW : 0u;  // the same on every thread
}

__global__ void __launch_bounds__(kPoolThreads) reserve_pages_kernel(const __grid_constant__ PoolParams p) {
  __shared__ int64_t sums[32];
  __shared__ uint32_t s_err;
  __shared__ int64_t s_free;
  __shared__ uint32_t s_rows[kRowBitmapWords];
  __shared__ int32_t s_lo, s_hi;
  pdl_wait();  // lengths may be written by the kernel just before this one
  if (threadIdx.x == 0) {
    s_err = 0;
    s_free = *p.free_count;
  }
  __syncthreads();
  const int64_t free_n = s_free;
  uint32_t err = 0;
  int64_t total = 0;
  for (int32_t base = 0; base < p.n; base += kPoolThreads) {
    const int32_t i = base + static_cast<int32_t>(threadIdx.x);
    int32_t row = 0;
    int64_t held = 0, lack = 0;
    if (i < p.n) err |= reserve_need(p, i, row, held, lack);
    int64_t t;
    block_exclusive_scan(lack, t, sums);
    total += t;
  }
  err |= duplicate_rows(p.rows, p.n, p.num_rows, s_rows, &s_lo, &s_hi);  // table_index; NULL: rows 0..n-1
  // the pool is checked only for valid inputs, then the ids about to leave
  // the list: free_pages[free_n - total, free_n)
  const bool inputs_ok = block_or(err, &s_err) == 0;
  const bool pool_ok = free_n >= 0 && free_n <= p.capacity && total <= free_n;
  if (inputs_ok && !pool_ok && threadIdx.x == 0) err |= YL_DEVERR_POOL_EMPTY;
  if (inputs_ok && pool_ok) {
    for (int64_t k = threadIdx.x; k < total; k += kPoolThreads)
      if (!page_ok(p.free_pages[free_n - total + k], p.capacity)) err |= YL_DEVERR_PAGE_RANGE;
  }
  if (block_or(err, &s_err) != 0) {
    if (threadIdx.x == 0) raise_deverr(p.error_word, s_err);
    return;
  }
  // sequence i takes free_pages[free_n - off_i - lack_i, free_n - off_i), in order
  int64_t running = 0;
  for (int32_t base = 0; base < p.n; base += kPoolThreads) {
    const int32_t i = base + static_cast<int32_t>(threadIdx.x);
    int32_t row = 0;
    int64_t held = 0, lack = 0;
    if (i < p.n) reserve_need(p, i, row, held, lack);
    int64_t t;
    const int64_t off = running + block_exclusive_scan(lack, t, sums);
    if (lack > 0) {
      const int32_t *src = p.free_pages + (free_n - off - lack);
      int32_t *dst = p.table + static_cast<int64_t>(row) * p.stride + held;
      for (int64_t j = 0; j < lack; ++j) dst[j] = src[j];
    }
    running += t;
  }
  if (threadIdx.x == 0) *p.free_count = static_cast<int32_t>(free_n - total);
}

__global__ void __launch_bounds__(kPoolThreads) release_pages_kernel(const __grid_constant__ PoolParams p) {
  __shared__ int64_t sums[32];
  __shared__ uint32_t s_err;
  __shared__ int64_t s_free;
  __shared__ uint32_t s_rows[kRowBitmapWords];
  __shared__ int32_t s_lo, s_hi;
  pdl_wait();
  if (threadIdx.x == 0) {
    s_err = 0;
    s_free = *p.free_count;
  }
  __syncthreads();
  const int64_t free_n = s_free;
  uint32_t err = 0;
  int64_t total = 0;
  for (int32_t base = 0; base < p.n; base += kPoolThreads) {
    const int32_t r = base + static_cast<int32_t>(threadIdx.x);
    int32_t row = 0;
    int64_t count = 0;
    if (r < p.n) {
      err |= release_count(p, r, row, count);
      const int32_t *ids = p.table + static_cast<int64_t>(row) * p.stride;
      for (int64_t j = 0; j < count; ++j)
        if (!page_ok(ids[j], p.capacity)) err |= YL_DEVERR_PAGE_RANGE;
    }
    int64_t t;
    block_exclusive_scan(count, t, sums);
    total += t;
  }
  err |= duplicate_rows(p.rows, p.n, p.num_rows, s_rows, &s_lo, &s_hi);
  // the free list is checked only for valid inputs
  if (block_or(err, &s_err) == 0 && threadIdx.x == 0 && (free_n < 0 || free_n + total > p.capacity))
    err |= YL_DEVERR_POOL_OVERFLOW;
  if (block_or(err, &s_err) != 0) {
    if (threadIdx.x == 0) raise_deverr(p.error_word, s_err);
    return;
  }
  // row r's pages go to free_pages[free_n + off_r, ...), in row order
  int64_t running = 0;
  for (int32_t base = 0; base < p.n; base += kPoolThreads) {
    const int32_t r = base + static_cast<int32_t>(threadIdx.x);
    int32_t row = 0;
    int64_t count = 0;
    if (r < p.n) release_count(p, r, row, count);
    int64_t t;
    const int64_t off = running + block_exclusive_scan(count, t, sums);
    if (count > 0) {
      int32_t *ids = p.table + static_cast<int64_t>(row) * p.stride;
      int32_t *dst = p.free_pages + free_n + off;
      for (int64_t j = 0; j < count; ++j) {
        dst[j] = ids[j];
        ids[j] = -1;
      }
    }
    running += t;
  }
  if (threadIdx.x == 0) *p.free_count = static_cast<int32_t>(free_n + total);
}

// Host checks shared by both entry points; the message names the caller.
int fail_in(const char *fn, int status, const char *fmt, long long a = 0, long long b = 0) {
  char buf[224];
  std::snprintf(buf, sizeof(buf), fmt, a, b);
  set_last_error(std::string(fn) + ": " + buf);
  return status;
}

int check_pool(const yl_page_pool &pool, const char *fn) {
  if (!pool.free_pages || !pool.free_count)
    return fail_in(fn, YL_ERR_NULL_ARG, "pool.free_pages and pool.free_count must be non-NULL");
  if (pool.capacity <= 0 || pool.capacity >= (1ll << 31))
    return fail_in(fn, YL_ERR_BAD_SIZE, "pool capacity=%lld must be in [1, 2^31)", pool.capacity);
  if ((reinterpret_cast<uintptr_t>(pool.free_pages) | reinterpret_cast<uintptr_t>(pool.free_count)) & 3u)
    return fail_in(fn, YL_ERR_ALIGNMENT, "pool arrays must be 4-byte aligned");
  return YL_OK;
}

int check_table(const char *fn, const int32_t *table, int64_t stride, int32_t num_rows, int32_t max_pages,
                int32_t page_size) {
  if (!table) return fail_in(fn, YL_ERR_NULL_ARG, "page_table must be non-NULL");
  if (page_size <= 0) return fail_in(fn, YL_ERR_BAD_SIZE, "page_size=%lld must be > 0", page_size);
  if (num_rows < 0 || max_pages < 0 || stride < max_pages)
    return fail_in(fn, YL_ERR_BAD_SIZE, "page table: rows=%lld, max_pages_per_row=%lld, or a stride below the row",
                   num_rows, max_pages);
  if (reinterpret_cast<uintptr_t>(table) & 3u) return fail_in(fn, YL_ERR_ALIGNMENT, "page_table must be 4-byte aligned");
  return YL_OK;
}

}  // namespace ylk

extern "C" int yl_reserve_pages(const yl_reserve_args *a, cudaStream_t stream) {
  using namespace ylk;
  clear_last_error();
  if (a == nullptr) return fail(YL_ERR_NULL_ARG, "yl_reserve_pages: args is NULL");
  if (a->batch_size < 0) return fail(YL_ERR_BAD_SIZE, "yl_reserve_pages: batch_size=%lld < 0", a->batch_size);
  if (a->batch_size == 0) return YL_OK;
  int st = check_pool(a->pool, "yl_reserve_pages");
  if (st == YL_OK)
    st = check_table("yl_reserve_pages", a->page_table, a->page_table_stride, a->num_table_rows, a->max_pages_per_row,
                     a->page_size);
  if (st != YL_OK) return st;
  if (!a->prior_len || !a->new_len) return fail(YL_ERR_NULL_ARG, "yl_reserve_pages: prior_len and new_len must be non-NULL");
  if ((reinterpret_cast<uintptr_t>(a->prior_len) | reinterpret_cast<uintptr_t>(a->new_len) |
       reinterpret_cast<uintptr_t>(a->table_index)) & 3u)
    return fail(YL_ERR_ALIGNMENT, "yl_reserve_pages: length arrays must be 4-byte aligned");
  if (a->table_index == nullptr && a->batch_size > a->num_table_rows)
    return fail(YL_ERR_BAD_SIZE, "yl_reserve_pages: batch_size=%lld rows without table_index exceed the table (%lld)",
                a->batch_size, a->num_table_rows);
  PoolParams p{a->pool.free_pages, a->pool.free_count, a->pool.capacity, a->page_table, a->prior_len, a->new_len,
               a->table_index, a->page_table_stride, a->num_table_rows, a->max_pages_per_row, a->page_size,
               a->batch_size, a->error_word};
  return launch_dependent(reserve_pages_kernel, dim3(1), dim3(kPoolThreads), 0, stream, "yl_reserve_pages launch", p);
}

extern "C" int yl_release_pages(const yl_release_args *a, cudaStream_t stream) {
  using namespace ylk;
  clear_last_error();
  if (a == nullptr) return fail(YL_ERR_NULL_ARG, "yl_release_pages: args is NULL");
  if (a->num_release < 0) return fail(YL_ERR_BAD_SIZE, "yl_release_pages: num_release=%lld < 0", a->num_release);
  if (a->num_release == 0) return YL_OK;
  int st = check_pool(a->pool, "yl_release_pages");
  if (st == YL_OK)
    st = check_table("yl_release_pages", a->page_table, a->page_table_stride, a->num_table_rows, a->max_pages_per_row,
                     a->page_size);
  if (st != YL_OK) return st;
  if (!a->rows || !a->num_tokens) return fail(YL_ERR_NULL_ARG, "yl_release_pages: rows and num_tokens must be non-NULL");
  if ((reinterpret_cast<uintptr_t>(a->rows) | reinterpret_cast<uintptr_t>(a->num_tokens)) & 3u)
    return fail(YL_ERR_ALIGNMENT, "yl_release_pages: rows and num_tokens must be 4-byte aligned");
  PoolParams p{a->pool.free_pages, a->pool.free_count, a->pool.capacity, a->page_table, a->num_tokens, nullptr,
               a->rows, a->page_table_stride, a->num_table_rows, a->max_pages_per_row, a->page_size,
               a->num_release, a->error_word};
  return launch_dependent(release_pages_kernel, dim3(1), dim3(kPoolThreads), 0, stream, "yl_release_pages launch", p);
}
