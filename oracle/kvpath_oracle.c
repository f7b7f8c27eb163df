/*
 * CPU oracle of the paged KV-cache store and the batch index build.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain C, what the
 * reference computes on this path; the tests compare the CUDA kernels with it
 * and bench.py times it as the CPU baseline.  No product code links it.
 *
 *   oracle_kv_store     follows StoreKVCacheKernel (src/kvcache/store_kv_cache.cu:60-72:
 *                       k_cache[indices[i]] <- k[i], v_cache[indices[i]] <- v[i], a
 *                       row of kElementSize bytes) as driven per layer by
 *                       MHAKVCache::StoreKV (src/include/kvcache/mha_kvcache.h:76-86,
 *                       N == 0 is a no-op), looped over layers.
 *   oracle_build_index  the page-array semantics that BatchManager::NextBatch
 *                       (src/include/batch/batch_manager.h:97-112) intends, per
 *                       request (table_index, cached_len, device_len), generalised
 *                       to page_size >= 1: load indices are the page-table row's
 *                       first ceil(device_len / page_size) entries and the new
 *                       tokens' slots are its entries at [cached_len, device_len).
 *                       Make2DIndices (batch_manager.h:30-51) drops the row stride
 *                       and stores indices in a float tensor; those defects are not
 *                       reproduced.
 *
 * Both functions take HOST pointers and the same argument meanings as the C
 * ABI in include/yl_kvpath.h, including its error-word bits, so that a test
 * can run the same case through both.  `threads` > 1 splits the store over
 * POSIX threads (duplicate slots within one call are then unordered, as on
 * the GPU); threads == 1 is strictly sequential (last writer wins).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <unistd.h>

#define ORACLE_SLOT_RANGE 0x1u
#define ORACLE_PAGE_RANGE 0x2u
#define ORACLE_ROW_OVERFLOW 0x4u
#define ORACLE_INDICES_CAP 0x8u
#define ORACLE_SLOTS_CAP 0x10u
#define ORACLE_NEGATIVE_LEN 0x20u
#define ORACLE_INDPTR_OVERFLOW 0x40u
#define ORACLE_TABLE_ROW 0x80u

static int64_t read_slot(const void *slots, int is64, int64_t i) {
  return is64 ? ((const int64_t *)slots)[i] : (int64_t)((const int32_t *)slots)[i];
}

typedef struct store_job {
  const uint8_t *k, *v;
  uint8_t *k_cache, *v_cache;
  const void *slots;
  int slot_is_int64;
  int64_t num_tokens, row_bytes, k_row_stride, v_row_stride, cache_row_stride;
  int64_t k_layer_stride, v_layer_stride, cache_layer_stride, num_slots;
  int64_t begin, end; /* rows [begin, end) of the (layer, token) space */
  int64_t copied;
  uint32_t err;
} store_job;

static void *store_range(void *arg) {
  store_job *j = (store_job *)arg;
  for (int64_t r = j->begin; r < j->end; ++r) {
    const int64_t layer = r / j->num_tokens;
    const int64_t i = r % j->num_tokens;
    const int64_t slot = read_slot(j->slots, j->slot_is_int64, i);
    if (slot < 0 || (j->num_slots > 0 && slot >= j->num_slots)) {
      if (slot != -1) j->err |= ORACLE_SLOT_RANGE;
      continue;
    }
    memcpy(j->k_cache + layer * j->cache_layer_stride + slot * j->cache_row_stride,
           j->k + layer * j->k_layer_stride + i * j->k_row_stride, (size_t)j->row_bytes);
    memcpy(j->v_cache + layer * j->cache_layer_stride + slot * j->cache_row_stride,
           j->v + layer * j->v_layer_stride + i * j->v_row_stride, (size_t)j->row_bytes);
    j->copied += 2;
  }
  return NULL;
}

#define ORACLE_MAX_THREADS 256

/* Returns the number of rows copied (K and V rows both counted). */
int64_t oracle_kv_store(const uint8_t *k, const uint8_t *v, uint8_t *k_cache, uint8_t *v_cache,
                        const void *slots, int slot_is_int64, int64_t num_tokens, int64_t row_bytes,
                        int64_t k_row_stride, int64_t v_row_stride, int64_t cache_row_stride, int32_t num_layers,
                        int64_t k_layer_stride, int64_t v_layer_stride, int64_t cache_layer_stride,
                        int64_t num_slots, uint32_t *error_word, int threads) {
  if (num_tokens <= 0 || num_layers <= 0) return 0;
  const int64_t total = (int64_t)num_layers * num_tokens;
  if (threads < 1) threads = 1;
  if (threads > ORACLE_MAX_THREADS) threads = ORACLE_MAX_THREADS;
  if (threads > total) threads = (int)total;
  store_job jobs[ORACLE_MAX_THREADS];
  pthread_t tids[ORACLE_MAX_THREADS];
  int started[ORACLE_MAX_THREADS];
  for (int t = 0; t < threads; ++t) {
    store_job j = {k, v, k_cache, v_cache, slots, slot_is_int64, num_tokens, row_bytes, k_row_stride,
                   v_row_stride, cache_row_stride, k_layer_stride, v_layer_stride, cache_layer_stride, num_slots,
                   total * t / threads, total * (t + 1) / threads, 0, 0};
    jobs[t] = j;
  }
  for (int t = 1; t < threads; ++t) started[t] = pthread_create(&tids[t], NULL, store_range, &jobs[t]) == 0;
  store_range(&jobs[0]);
  for (int t = 1; t < threads; ++t) {
    if (started[t]) pthread_join(tids[t], NULL);
    else store_range(&jobs[t]);
  }
  int64_t copied = 0;
  uint32_t err = 0;
  for (int t = 0; t < threads; ++t) {
    copied += jobs[t].copied;
    err |= jobs[t].err;
  }
  if (error_word) *error_word |= err;
  return copied;
}

/*
 * Index build.  All arrays are host arrays; outputs may be NULL except
 * kv_indptr and qo_indptr.  Slot entries past the batch's new tokens, up to
 * slot_capacity, are set to -1.  Returns 0, or -1 when a running sum passes
 * INT32_MAX (outputs other than the error word are then unspecified).
 */
int oracle_build_index(const int32_t *prior_len, const int32_t *new_len, const int32_t *page_table,
                       const int32_t *table_index, int64_t page_table_stride, int32_t num_table_rows,
                       int32_t max_pages_per_row, int32_t page_size, int32_t batch_size, int64_t num_pages,
                       int32_t *kv_indptr, int32_t *kv_indices, int32_t *kv_last_page_len, int32_t *qo_indptr,
                       void *slot_mapping, int slot_is_int64, int64_t kv_indices_capacity, int64_t slot_capacity,
                       uint32_t *error_word) {
  uint32_t err = 0;
  int64_t kv_off = 0, qo_off = 0;
  int rc = 0;
  if (!kv_indices) kv_indices_capacity = 0;
  if (!slot_mapping) slot_capacity = 0;
  kv_indptr[0] = 0;
  qo_indptr[0] = 0;
  for (int32_t i = 0; i < batch_size; ++i) {
    int32_t prior = prior_len[i];
    int32_t fresh = new_len[i];
    if (prior < 0 || fresh < 0) {
      err |= ORACLE_NEGATIVE_LEN;
      if (prior < 0) prior = 0;
      if (fresh < 0) fresh = 0;
    }
    int32_t row = i;
    int row_ok = 1;
    if (table_index) {
      row = table_index[i];
      if (row < 0 || row >= num_table_rows) {
        err |= ORACLE_TABLE_ROW;
        row_ok = 0;
      }
    }
    const int64_t total = (int64_t)prior + fresh;
    int64_t pages = row_ok ? (total + page_size - 1) / page_size : 0;
    if (pages > max_pages_per_row) {
      err |= ORACLE_ROW_OVERFLOW;
      pages = max_pages_per_row;
    }
    const int32_t *prow = page_table ? page_table + (int64_t)row * page_table_stride : 0;
    /* kv_indices: the row's first `pages` entries */
    for (int64_t j = 0; j < pages; ++j) {
      const int64_t e = kv_off + j;
      if (e >= kv_indices_capacity) break;
      const int32_t page = prow[j];
      if (num_pages > 0 && (page < 0 || page >= num_pages)) err |= ORACLE_PAGE_RANGE;
      kv_indices[e] = page;
    }
    /* slot_mapping: one slot per new token */
    for (int64_t t = 0; t < fresh; ++t) {
      const int64_t e = qo_off + t;
      if (e >= slot_capacity) break;
      const int64_t pos = prior + t;
      const int64_t pidx = pos / page_size;
      int64_t slot = -1;
      /* positions at or past 2^31 get no slot (the kernel's 32-bit divider) */
      if (pos <= INT32_MAX && pidx < pages) {
        const int32_t page = prow[pidx];
        const int in_range = page >= 0 && (num_pages <= 0 || page < num_pages);
        const int64_t s = (int64_t)page * page_size + pos % page_size;
        if (in_range && (slot_is_int64 || s <= INT32_MAX)) slot = s;
        else err |= ORACLE_PAGE_RANGE;
      }
      if (slot_is_int64) ((int64_t *)slot_mapping)[e] = slot;
      else ((int32_t *)slot_mapping)[e] = (int32_t)slot;
    }
    if (kv_last_page_len) kv_last_page_len[i] = pages == 0 ? 0 : (int32_t)((total - 1) % page_size + 1);
    kv_off += pages;
    qo_off += fresh;
    if (kv_off > INT32_MAX || qo_off > INT32_MAX) {
      err |= ORACLE_INDPTR_OVERFLOW;
      rc = -1;
      break;
    }
    kv_indptr[i + 1] = (int32_t)kv_off;
    qo_indptr[i + 1] = (int32_t)qo_off;
  }
  /* slot entries past the batch's tokens, up to the capacity, hold -1 */
  for (int64_t e = qo_off; rc == 0 && e < slot_capacity; ++e) {
    if (slot_is_int64) ((int64_t *)slot_mapping)[e] = -1;
    else ((int32_t *)slot_mapping)[e] = -1;
  }
  if (kv_off > kv_indices_capacity && kv_indices) err |= ORACLE_INDICES_CAP;
  if (qo_off > slot_capacity && slot_mapping) err |= ORACLE_SLOTS_CAP;
  if (error_word) *error_word |= err;
  return rc;
}

/*
 * Row gather: out[i] <- table[indices[i]], following IndexKernel
 * (src/layers/index.cu:61-72: dst row i gets weights row indices[i]) with
 * byte strides; an index outside [0, num_rows) (when num_rows > 0) or
 * negative zero-fills its row, -1 silently, others also set bit 0x400.
 * Returns the rows copied from the table.
 */
#define ORACLE_INDEX_RANGE 0x400u
int64_t oracle_gather_rows(const uint8_t *table, uint8_t *out, const void *indices, int index_is_int64,
                           int64_t num_indices, int64_t row_bytes, int64_t table_row_stride, int64_t out_row_stride,
                           int64_t num_rows, uint32_t *error_word) {
  int64_t copied = 0;
  uint32_t err = 0;
  for (int64_t i = 0; i < num_indices; ++i) {
    const int64_t r = read_slot(indices, index_is_int64, i);
    uint8_t *dst = out + i * out_row_stride;
    if (r < 0 || (num_rows > 0 && r >= num_rows)) {
      if (r != -1) err |= ORACLE_INDEX_RANGE;
      memset(dst, 0, (size_t)row_bytes);
      continue;
    }
    memcpy(dst, table + r * table_row_stride, (size_t)row_bytes);
    ++copied;
  }
  if (error_word) *error_word |= err;
  return copied;
}

/*
 * Page allocator, request by request as KVCacheManager::AllocateIndices runs
 * (src/include/kvcache/cache_manager.h:119-131): a request lacking `size`
 * pages takes the last `size` entries of the free list, in order, and the
 * list keeps the rest (the reference keeps slice(0, size), a defect); the
 * pages go into the request's page-table row after the pages it holds
 * (WritePageTable, :148-155, meant for the page table).  All-or-nothing:
 * returns error bits and changes nothing when any request is invalid (a
 * page-table row named twice included) or the list is short.  Bits as in
 * yl_kvpath.h.
 */
#define O_NEGATIVE_LEN 0x20u
#define O_TABLE_ROW 0x80u
#define O_ROW_OVERFLOW 0x4u
#define O_PAGE_RANGE 0x2u
#define O_POOL_EMPTY 0x1000u
#define O_POOL_OVERFLOW 0x2000u
#define O_DUPLICATE_ROW 0x4000u

/* 0x4000 when a valid row in [0, num_rows) appears twice in rows[0, n):
 * two sequences of one call would write one page-table row (reserve), or one
 * row's pages would enter the free list twice (release). */
static uint32_t o_duplicate_rows(const int32_t *rows, int32_t n, int32_t num_rows) {
  if (rows == NULL || n < 2 || num_rows <= 0) return 0;
  unsigned char *seen = (unsigned char *)calloc((size_t)num_rows, 1);
  uint32_t err = 0;
  for (int32_t i = 0; seen && i < n && !err; ++i) {
    const int32_t r = rows[i];
    if (r < 0 || r >= num_rows) continue;
    if (seen[r]) err = O_DUPLICATE_ROW;
    seen[r] = 1;
  }
  free(seen);
  return err;
}

static int64_t o_pages_for(int64_t tokens, int32_t ps) { return (tokens + ps - 1) / ps; }

uint32_t oracle_reserve_pages(int32_t *free_pages, int32_t *free_count, int64_t capacity, int32_t *table,
                              int64_t stride, int32_t num_rows, int32_t max_pages, const int32_t *prior,
                              const int32_t *fresh, const int32_t *table_index, int32_t page_size, int32_t batch) {
  uint32_t err = 0;
  int64_t total = 0;
  for (int32_t i = 0; i < batch; ++i) {
    const int32_t row = table_index ? table_index[i] : i;
    if (prior[i] < 0 || fresh[i] < 0) { err |= O_NEGATIVE_LEN; continue; }
    if (row < 0 || row >= num_rows) { err |= O_TABLE_ROW; continue; }
    const int64_t need = o_pages_for((int64_t)prior[i] + fresh[i], page_size);
    if (need > max_pages) { err |= O_ROW_OVERFLOW; continue; }
    total += need - o_pages_for(prior[i], page_size);
  }
  err |= o_duplicate_rows(table_index, batch, num_rows);
  const int64_t n = *free_count;
  if (!err && (n < 0 || n > capacity || total > n)) err |= O_POOL_EMPTY;
  for (int64_t k = n - total; !err && k < n; ++k)
    if (free_pages[k] < 0 || free_pages[k] >= capacity) err |= O_PAGE_RANGE;
  if (err) return err;
  int64_t top = n;
  for (int32_t i = 0; i < batch; ++i) {
    const int32_t row = table_index ? table_index[i] : i;
    const int64_t held = o_pages_for(prior[i], page_size);
    const int64_t lack = o_pages_for((int64_t)prior[i] + fresh[i], page_size) - held;
    for (int64_t j = 0; j < lack; ++j) table[row * stride + held + j] = free_pages[top - lack + j];
    top -= lack;
  }
  *free_count = (int32_t)top;
  return 0;
}

/* Release: rows in order append their ceil(tokens / page_size) pages to the
 * free list and clear those table entries to -1; all-or-nothing (a row named
 * twice is invalid). */
uint32_t oracle_release_pages(int32_t *free_pages, int32_t *free_count, int64_t capacity, int32_t *table,
                              int64_t stride, int32_t num_rows, int32_t max_pages, const int32_t *rows,
                              const int32_t *num_tokens, int32_t page_size, int32_t count) {
  uint32_t err = 0;
  int64_t total = 0;
  for (int32_t r = 0; r < count; ++r) {
    if (num_tokens[r] < 0) { err |= O_NEGATIVE_LEN; continue; }
    if (rows[r] < 0 || rows[r] >= num_rows) { err |= O_TABLE_ROW; continue; }
    const int64_t c = o_pages_for(num_tokens[r], page_size);
    if (c > max_pages) { err |= O_ROW_OVERFLOW; continue; }
    for (int64_t j = 0; j < c; ++j) {
      const int32_t id = table[rows[r] * stride + j];
      if (id < 0 || id >= capacity) err |= O_PAGE_RANGE;
    }
    total += c;
  }
  err |= o_duplicate_rows(rows, count, num_rows);
  const int64_t n = *free_count;
  if (!err && (n < 0 || n + total > capacity)) err |= O_POOL_OVERFLOW;
  if (err) return err;
  int64_t top = n;
  for (int32_t r = 0; r < count; ++r) {
    const int64_t c = o_pages_for(num_tokens[r], page_size);
    for (int64_t j = 0; j < c; ++j) {
      free_pages[top++] = table[rows[r] * stride + j];
      table[rows[r] * stride + j] = -1;
    }
  }
  *free_count = (int32_t)top;
  return 0;
}

/*
 * Range expansion, following Make2DIndices (src/include/batch/batch_manager.h:30-51):
 * for each range {row, col_start, col_end} in order, the indices
 * row + col_start .. row + col_end - 1 (batch_manager.h:42-47), concatenated,
 * as int64 instead of the helper's float.  Validation as in yl_make_2d_indices:
 * a negative entry or col_end < col_start adds nothing (bit 0x20); row +
 * col_end past INT64_MAX adds nothing (bit 0x400); lengths count at most 2^40;
 * indices past `capacity` are not written (bit 0x8).  *count gets the total.
 */
uint32_t oracle_make_2d_indices(const int64_t *ranges, int64_t num_ranges, int64_t *out, int64_t capacity,
                                int64_t *count) {
  uint32_t err = 0;
  int64_t pos = 0;
  for (int64_t r = 0; r < num_ranges; ++r) {
    const int64_t row = ranges[3 * r], lo = ranges[3 * r + 1], hi = ranges[3 * r + 2];
    if (row < 0 || lo < 0 || hi < lo) { err |= ORACLE_NEGATIVE_LEN; continue; }
    if (row > INT64_MAX - hi) { err |= ORACLE_INDEX_RANGE; continue; }
    const int64_t len = hi - lo < ((int64_t)1 << 40) ? hi - lo : ((int64_t)1 << 40);
    for (int64_t c = 0; c < len && pos + c < capacity; ++c) out[pos + c] = row + lo + c;
    pos += len;
  }
  if (pos > capacity) err |= ORACLE_INDICES_CAP;
  if (count) *count = pos;
  return err;
}

/* Host threads available to this process (online processors). */
int oracle_max_threads(void) {
  const long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}
