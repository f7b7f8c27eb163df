/*
 * yl_kvpath.h — C ABI of the B200 paged KV-cache store and batch index build.
 *
 * Two hot operations of an LLM serving step, as hand-written sm_100a CUDA:
 *
 *   yl_kv_store     scatter each step's new K/V rows into the paged pool by
 *                   slot mapping (replaces yllang::StoreKVCache,
 *                   src/kvcache/store_kv_cache.cu:95-163, declared at
 *                   src/include/kvcache/store_kv_cache.h:29-31, and the call in
 *                   MHAKVCache::StoreKV, src/include/kvcache/mha_kvcache.h:76-86).
 *
 *   yl_build_index  build the paged-attention page arrays of one batch
 *                   (kv_indptr, kv_indices, kv_last_page_len, qo_indptr,
 *                   slot_mapping) from per-sequence lengths and page-table rows
 *                   (replaces the load/write index construction of
 *                   BatchManager::NextBatch, src/include/batch/batch_manager.h:83-115,
 *                   and Make2DIndices, batch_manager.h:30-51).
 *
 * Every pointer in an argument struct is a DEVICE pointer unless stated
 * otherwise; every stride and size is in BYTES unless its name says
 * "elements".  Calls are asynchronous on the given stream (NULL = legacy
 * default stream), allocate nothing and never synchronise.  A call returns
 * YL_OK or a negative yl_status; no C++ exception crosses this boundary.
 * Argument errors are detected on the host before any launch.  Data errors
 * that only the device can see (a slot or page id out of range, a page-table
 * row too short, an output buffer too small) skip the offending element and
 * set a bit in the caller's optional device error word (see YL_DEVERR_*);
 * kernels never trap.
 *
 * Stream order is that of plain launches.  Most kernels here are launched as
 * programmatic dependents of the kernel before them on the stream, which
 * lets their blocks be placed while that kernel drains; each waits for that
 * kernel to complete before touching memory it may have written.  The one
 * exception, yl_kv_store, is a plain launch (it starts loading its K/V rows
 * at once).
 */
#ifndef YL_KVPATH_H_
#define YL_KVPATH_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as the CUDA runtime's cudaStream_t (an opaque CUstream_st*). */
struct CUstream_st;
typedef struct CUstream_st *cudaStream_t;

#define YL_KVPATH_ABI_VERSION 1

#if defined(__GNUC__)
#define YL_API __attribute__((visibility("default")))
#else
#define YL_API
#endif

/* Host-side status codes returned by every entry point. */
typedef enum yl_status {
  YL_OK = 0,
  YL_ERR_NULL_ARG = -1,     /* a required pointer is NULL                        */
  YL_ERR_BAD_SIZE = -2,     /* negative count, zero/negative row size, ...       */
  YL_ERR_ALIGNMENT = -3,    /* pointer/stride not a multiple of the element unit */
  YL_ERR_UNSUPPORTED = -4,  /* a combination this library does not implement     */
  YL_ERR_CUDA = -5          /* the CUDA runtime refused the launch               */
} yl_status;

/* Bits a kernel ORs into the caller's device error word. */
#define YL_DEVERR_SLOT_RANGE      0x1u  /* store: slot >= num_slots or < -1 (row skipped)   */
#define YL_DEVERR_PAGE_RANGE      0x2u  /* index: page id outside [0, num_pages)            */
#define YL_DEVERR_ROW_OVERFLOW    0x4u  /* index: a sequence needs more pages than its row  */
#define YL_DEVERR_INDICES_CAP     0x8u  /* index, ranges: output exceeds its capacity       */
#define YL_DEVERR_SLOTS_CAP       0x10u /* index: sum of new tokens exceeds slot_capacity   */
#define YL_DEVERR_NEGATIVE_LEN    0x20u /* index, ranges: a negative length (treated as 0)  */
#define YL_DEVERR_INDPTR_OVERFLOW 0x40u /* index: a running sum passed INT32_MAX (no fill)  */
#define YL_DEVERR_TABLE_ROW       0x80u /* index: table_index outside [0, num_table_rows)   */
#define YL_DEVERR_TOKEN_COUNT     0x100u /* step: sum of new_len differs from num_tokens      */
#define YL_DEVERR_TIMEOUT         0x200u /* store: a bulk copy did not complete within 2 s    */
#define YL_DEVERR_INDEX_RANGE     0x400u /* gather: index outside [-1, num_rows); ranges: index past INT64_MAX */
#define YL_DEVERR_POSITION_RANGE  0x800u /* qkv store: position outside [0, max_position)     */
#define YL_DEVERR_POOL_EMPTY      0x1000u /* reserve: fewer free pages than the batch needs  */
#define YL_DEVERR_POOL_OVERFLOW   0x2000u /* release: more pages than the free list holds    */
#define YL_DEVERR_DUPLICATE_ROW   0x4000u /* reserve, release: one table row named twice     */

/*
 * Store (replaces yllang::StoreKVCache<kElementSize>,
 * src/kvcache/store_kv_cache.cu:95-163, and its kernel StoreKVCacheKernel,
 * store_kv_cache.cu:46-77).
 *
 * For every layer l < num_layers and token i < num_tokens:
 *     row(k_cache, l, slots[i]) <- row(k, l, i)
 *     row(v_cache, l, slots[i]) <- row(v, l, i)
 * where row(base, l, r) is the row_bytes bytes at
 *     base + l * <layer stride> + r * <row stride>.
 * The copy is bit-exact and dtype-agnostic.  With num_layers == 1 this is the
 * reference's per-layer call; num_layers > 1 stores every layer of one step in
 * one launch (inputs laid out [L, N, row] with the given strides, pool laid
 * out layer-major as MHAKVCache allocates it, mha_kvcache.h:42-62).
 *
 * Slots are int32 or int64 (slot_is_int64).  The reference always reads
 * int64 (store_kv_cache.cu:127 compares bytes with bits); here both work.
 * A slot of -1 marks a padding token and is skipped silently.  When
 * num_slots > 0, a slot outside [-1, num_slots) skips its row and sets
 * YL_DEVERR_SLOT_RANGE.  Duplicate slots inside one call are outside the
 * contract (as in the reference, the winner is unspecified); across calls on
 * one stream the later call wins.  num_tokens == 0 is a no-op
 * (mha_kvcache.h:77-79).
 *
 * Alignment: the widest unit u in {16, 8, 4, 2, 1} bytes that divides
 * row_bytes, every base pointer and every stride is used; the fast paths need
 * u == 16 (bf16/fp16 rows of H*D a multiple of 8 elements, fp32 of 4).
 */
typedef struct yl_store_args {
  const void *k;              /* input K rows of layer 0                          */
  const void *v;              /* input V rows of layer 0                          */
  void *k_cache;              /* K pool of layer 0, viewed as [num_slots, row]    */
  void *v_cache;              /* V pool of layer 0                                */
  const void *slots;          /* [num_tokens] int32 or int64 slot mapping          */
  int32_t slot_is_int64;      /* 0: int32 slots, 1: int64 slots                   */
  int32_t num_layers;         /* >= 1                                             */
  int64_t num_tokens;         /* >= 0                                             */
  int64_t row_bytes;          /* bytes of one token's row (H_local*D*dtype size)  */
  int64_t k_row_stride;       /* bytes between consecutive tokens of k            */
  int64_t v_row_stride;       /* bytes between consecutive tokens of v            */
  int64_t cache_row_stride;   /* bytes between consecutive slots of either pool   */
  int64_t k_layer_stride;     /* bytes between layers of k (ignored if L == 1)    */
  int64_t v_layer_stride;     /* bytes between layers of v                        */
  int64_t cache_layer_stride; /* bytes between layers of either pool              */
  int64_t num_slots;          /* slots per layer for range checks; <= 0: no check */
  uint32_t *error_word;       /* optional device word for YL_DEVERR_* bits        */
} yl_store_args;

YL_API int yl_kv_store(const yl_store_args *args, cudaStream_t stream);

/*
 * Index build (replaces the index construction of BatchManager::NextBatch,
 * src/include/batch/batch_manager.h:83-115, and Make2DIndices,
 * batch_manager.h:30-51, generalised from page_size 1 to any page size; the
 * output is the paged-KV page-table format a flashinfer paged-attention
 * call consumes).
 *
 * Per sequence i < batch_size, with row_i = table_index ? table_index[i] : i,
 * P_i[j] = page_table[row_i * page_table_stride + j], total_i =
 * prior_len[i] + new_len[i] and np_i = ceil(total_i / page_size):
 *     kv_indptr[0] = 0,  kv_indptr[i+1] = kv_indptr[i] + np_i
 *     kv_indices[kv_indptr[i] + j] = P_i[j]                  (j < np_i)
 *     kv_last_page_len[i] = (total_i - 1) % page_size + 1    (0 if total_i == 0)
 *     qo_indptr[0] = 0,  qo_indptr[i+1] = qo_indptr[i] + new_len[i]
 *     slot_mapping[qo_indptr[i] + t] = P_i[p / page_size] * page_size + p % page_size,
 *         p = prior_len[i] + t                               (t < new_len[i])
 * prior_len plays the role of Request::CachedLen and prior_len + new_len of
 * Request::DeviceLen (src/include/request/request.h:81-92).
 *
 * Checks on the device (each skips the element and sets its error bit):
 * np_i > max_pages_per_row (the sequence keeps max_pages_per_row pages and
 * its slots past them are written as -1), page ids outside [0, num_pages)
 * when num_pages > 0 (kv_indices keeps the id, the slot is written as -1),
 * table_index outside [0, num_table_rows) (the sequence gets no pages and
 * -1 slots), sum of np_i > kv_indices_capacity, sum of new_len >
 * slot_capacity, negative lengths (treated as 0).  slot_mapping entries past
 * qo_indptr[B], up to slot_capacity, are set to -1 (padding), so a store
 * given the whole buffer skips them.
 * Any outputs except kv_indptr/qo_indptr may be NULL to skip them.
 */
typedef struct yl_index_args {
  const int32_t *prior_len;     /* [B] tokens already in the pool               */
  const int32_t *new_len;       /* [B] tokens stored this step                  */
  const int32_t *page_table;    /* 2-D page table, int32 page ids               */
  const int32_t *table_index;   /* [B] page-table row per sequence, or NULL     */
  int64_t page_table_stride;    /* ELEMENTS between page-table rows             */
  int32_t num_table_rows;       /* rows of page_table; > 0 required with        */
                                /* table_index; without it rows 0..B-1 are used */
                                /* (checked against this count when > 0)        */
  int32_t max_pages_per_row;    /* page-table columns usable by a sequence      */
  int32_t page_size;            /* tokens per page, >= 1                        */
  int32_t batch_size;           /* B >= 0                                       */
  int32_t slot_is_int64;        /* element type of slot_mapping                 */
  int64_t num_pages;            /* pool pages for range checks; <= 0: no check  */
  int32_t *kv_indptr;           /* [B+1]                                        */
  int32_t *kv_indices;          /* [kv_indices_capacity]                        */
  int32_t *kv_last_page_len;    /* [B]                                          */
  int32_t *qo_indptr;           /* [B+1]                                        */
  void *slot_mapping;           /* [slot_capacity] int32 or int64               */
  int64_t kv_indices_capacity;  /* elements available in kv_indices             */
  int64_t slot_capacity;        /* elements available in slot_mapping           */
  uint32_t *error_word;         /* optional device word for YL_DEVERR_* bits    */
} yl_index_args;

/*
 * Stream order: the index kernel is launched as a programmatic dependent of
 * the kernel before it on the stream (its blocks may be placed while that
 * kernel drains) and waits for that kernel to complete before it reads any
 * input, so the call observes every earlier write on the stream, as a plain
 * launch does.  (A preceding kernel that was itself launched as a
 * programmatic dependent must, as that contract requires of it, wait for its
 * own predecessor before completing.)
 */
YL_API int yl_build_index(const yl_index_args *args, cudaStream_t stream);

/*
 * Step: yl_build_index(&index) followed by yl_kv_store of every layer with
 * slots = index.slot_mapping, as two launches that overlap: the store starts
 * loading its K/V rows while the index build runs, and for a decode batch
 * (store.num_tokens == batch_size, every new_len 1) computes its slots
 * itself instead of waiting for them.  The result is identical to the two
 * calls.
 * This is one serving step of the reference's path: the per-step index work
 * of BatchManager::NextBatch (src/include/batch/batch_manager.h:97-112)
 * followed by MHAKVCache::StoreKV (src/include/kvcache/mha_kvcache.h:76-86)
 * for every layer.
 *
 * index.slot_mapping is required, with slot_capacity >= store.num_tokens;
 * store.slots, store.slot_is_int64 and store.error_word are ignored (the
 * slots are index.slot_mapping, errors go to index.error_word).
 * store.num_tokens must equal the sum of new_len (else
 * YL_DEVERR_TOKEN_COUNT; tokens without a sequence are not stored).
 */
typedef struct yl_step_args {
  yl_index_args index;
  yl_store_args store;
} yl_step_args;

YL_API int yl_kv_step(const yl_step_args *args, cudaStream_t stream);

/*
 * Row gather (replaces yllang::Index<kElementSize>, src/layers/index.cu:93-146,
 * and its kernel IndexKernel, index.cu:49-77, used by VocabEmbeddingLayer,
 * src/include/layers/vocab_embedding_layer.h:40-45): for i < num_indices,
 *     row(out, i) <- row(table, indices[i])
 * on the same copy engine as the store, with byte strides (the reference
 * passes the table's row stride in elements where it adds bytes,
 * index.cu:67,132).  An index outside [0, num_rows) zero-fills its output
 * row; -1 does so silently, anything else also sets YL_DEVERR_INDEX_RANGE
 * (when num_rows > 0; with num_rows <= 0 only negative indices are caught).
 */
typedef struct yl_gather_args {
  const void *table;          /* source rows, [num_rows, row]                     */
  void *out;                  /* destination rows, [num_indices, row]             */
  const void *indices;        /* [num_indices] int32 or int64                     */
  int32_t index_is_int64;
  int32_t reserved;           /* must be 0                                        */
  int64_t num_indices;
  int64_t row_bytes;
  int64_t table_row_stride;   /* bytes between table rows                         */
  int64_t out_row_stride;     /* bytes between output rows                        */
  int64_t num_rows;           /* table rows for range checks; <= 0: no check      */
  uint32_t *error_word;
} yl_gather_args;

YL_API int yl_gather_rows(const yl_gather_args *args, cudaStream_t stream);

/*
 * One layer's attention input, fused: per-head RMSNorm of Q and K, rotary
 * embedding of Q and K, then Q written out and K/V stored into the pool by
 * slot, reading every input row once.  Replaces the sequence the reference's
 * attention layer is built for (src/include/layers/attention.h:22-68): Q/K
 * RMSNorm through flashinfer::norm::QKRMSNorm (src/layers/rsm_norm.cu:35-52,
 * out = x * rsqrt(mean(x^2) + eps) * w over head_dim, fp32 arithmetic),
 * rotary embedding at the model config's rope_theta
 * (src/models/model_config.cpp:38) and StoreKVCache of K and V.  For token i
 * and head h (rows of head_dim elements):
 *     x  = q[i, h]            (or k[i, h])
 *     x  = T(x * rsqrt(sum(x^2) / head_dim + eps) * w)      if w != NULL
 *     x  = rotate(x, cos_sin_cache[positions[i]])           if cache != NULL
 *     q_out[i, h] = T(x);  k_cache[slots[i], h] = T(x);  v_cache[slots[i], h] = v[i, h]
 * The norm output is rounded to T before the rotation, as the unfused
 * norm-then-rope sequence stores it.  rotate: neox halves (element j pairs
 * with j + head_dim/2) or, with rope_interleaved, GPT-J pairs (2j, 2j+1);
 * cos_sin_cache[p] holds head_dim/2 cosines then head_dim/2 sines (fp32), the
 * layout of flashinfer's apply_rope_with_cos_sin_cache.  Slot -1 skips the
 * token's K/V rows silently, other out-of-range slots set
 * YL_DEVERR_SLOT_RANGE; a position outside [0, max_position) sets
 * YL_DEVERR_POSITION_RANGE and leaves that token's Q, K and V rows unwritten.
 * head_dim is 64, 128 or 256; T is bf16 or fp16.  No counterpart kernel in
 * the reference (its attention forward is a placeholder, attention.h:55).
 */
#define YL_DTYPE_BF16 0
#define YL_DTYPE_F16  1
typedef struct yl_qkv_store_args {
  const void *q;              /* [N, num_q_heads, head_dim] rows, q_row_stride apart   */
  const void *k;              /* [N, num_kv_heads, head_dim]                           */
  const void *v;              /* [N, num_kv_heads, head_dim]                           */
  void *q_out;                /* [N, num_q_heads, head_dim]; may equal q               */
  void *k_cache;              /* pool rows [num_slots, num_kv_heads * head_dim]        */
  void *v_cache;
  const void *slots;          /* [N] int32 or int64                                    */
  const void *q_weight;       /* [head_dim] RMSNorm weight of Q (type T); NULL: none   */
  const void *k_weight;       /* [head_dim] RMSNorm weight of K; NULL: none            */
  const float *cos_sin_cache; /* [max_position, head_dim] fp32; NULL: no rotation      */
  const void *positions;      /* [N] int32 or int64 (needed with cos_sin_cache)        */
  int32_t dtype;              /* YL_DTYPE_BF16 or YL_DTYPE_F16                         */
  int32_t slot_is_int64;
  int32_t position_is_int64;
  int32_t rope_interleaved;   /* 0: neox halves, 1: GPT-J pairs                        */
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  float eps;
  int64_t num_tokens;
  int64_t q_row_stride;       /* bytes between tokens of q                             */
  int64_t k_row_stride;
  int64_t v_row_stride;
  int64_t q_out_row_stride;
  int64_t cache_row_stride;   /* bytes between pool rows                               */
  int64_t num_slots;          /* pool rows for range checks; <= 0: no check            */
  int64_t max_position;       /* rows of cos_sin_cache                                 */
  uint32_t *error_word;
} yl_qkv_store_args;

YL_API int yl_qkv_norm_rope_store(const yl_qkv_store_args *args, cudaStream_t stream);

/*
 * Device page allocator: KVCacheManager's free-page list
 * (src/include/kvcache/cache_manager.h:105-131, AllocateIndices) and page
 * table (WritePageTable, :148-155) kept on the device, so the page ids the
 * index build reads never cross to the host.
 *
 * The pool: free_pages[0, *free_count) are the free page ids, a stack whose
 * top is the end.  Reserve gives the sequences of a batch, in batch order,
 * the pages they lack, each taking the current tail of the list in order
 * (AllocateIndices returns m_pages_.slice(0, -size), cache_manager.h:121-123,
 * the list keeping its head), and writes them into the sequences' page-table
 * rows after the pages already there: sequence i holds ceil(prior_len[i] /
 * page_size) pages and needs ceil((prior_len[i] + new_len[i]) / page_size).
 * Release appends the pages of the given rows (ceil(num_tokens[r] /
 * page_size) each, in row order) to the list and sets those table entries to
 * -1.  Both are all-or-nothing: any bad input (negative length, row outside
 * the table, one row named twice in the call, more pages than a row holds, a
 * page id outside [0, capacity)) or a pool that cannot satisfy the call sets
 * an error bit and changes nothing.  One CTA runs each call; calls on one stream are ordered, calls on
 * different streams on one pool race.  No counterpart kernel in the
 * reference, whose allocator is host code.
 */
typedef struct yl_page_pool {
  int32_t *free_pages;        /* [capacity] free page ids                          */
  int32_t *free_count;        /* one int32 on the device                           */
  int64_t capacity;           /* pages in the pool = entries of free_pages         */
} yl_page_pool;

typedef struct yl_reserve_args {
  yl_page_pool pool;
  int32_t *page_table;        /* [num_table_rows, page_table_stride] int32         */
  const int32_t *prior_len;   /* [batch_size] tokens already in the row's pages    */
  const int32_t *new_len;     /* [batch_size] tokens this step adds                */
  const int32_t *table_index; /* [batch_size] row of each sequence; NULL: row i    */
  int64_t page_table_stride;
  int32_t num_table_rows;
  int32_t max_pages_per_row;
  int32_t page_size;
  int32_t batch_size;
  uint32_t *error_word;
} yl_reserve_args;

YL_API int yl_reserve_pages(const yl_reserve_args *args, cudaStream_t stream);

typedef struct yl_release_args {
  yl_page_pool pool;
  int32_t *page_table;
  const int32_t *rows;        /* [num_release] rows to free                        */
  const int32_t *num_tokens;  /* [num_release] tokens each row holds               */
  int64_t page_table_stride;
  int32_t num_table_rows;
  int32_t max_pages_per_row;
  int32_t page_size;
  int32_t num_release;
  uint32_t *error_word;
} yl_release_args;

YL_API int yl_release_pages(const yl_release_args *args, cudaStream_t stream);

/*
 * Range expansion (replaces Make2DIndices, src/include/batch/batch_manager.h:30-51,
 * the helper NextBatch calls to turn {row, col_start, col_end} ranges into flat
 * page-table indices, batch_manager.h:97-107): for each range r in order,
 *     indices <- row_r + c   for c in [col_start_r, col_end_r)
 * concatenated, as int64 (the reference returns a default float tensor,
 * batch_manager.h:38, exact only below 2^24).  As in the reference, the row
 * entry is added as given: a caller that wants row-major flat indices passes
 * row * row_stride.  A range with a negative entry or col_end < col_start adds
 * nothing and sets YL_DEVERR_NEGATIVE_LEN; one whose last index would pass
 * INT64_MAX adds nothing and sets YL_DEVERR_INDEX_RANGE.  Indices past
 * indices_capacity are not written and set YL_DEVERR_INDICES_CAP; *count (when
 * given) receives the full total, so a caller can size the output first.
 */
typedef struct yl_ranges_args {
  const int64_t *ranges;      /* [num_ranges, 3] int64: row, col_start, col_end   */
  int64_t *indices;           /* [indices_capacity] int64 output                   */
  int64_t *count;             /* optional [1]: total indices of the valid ranges   */
  int64_t num_ranges;         /* <= 2^22                                           */
  int64_t indices_capacity;   /* < 2^40                                            */
  uint32_t *error_word;
} yl_ranges_args;

YL_API int yl_make_2d_indices(const yl_ranges_args *args, cudaStream_t stream);

/* Human-readable name of a yl_status value (static storage). */
YL_API const char *yl_status_string(int status);

/* Detail of the last failing call on this host thread ("" if none). */
YL_API const char *yl_last_error(void);

/* YL_KVPATH_ABI_VERSION of the loaded library. */
YL_API int yl_abi_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* YL_KVPATH_H_ */
