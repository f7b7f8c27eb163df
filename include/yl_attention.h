/*
 * yl_attention.h — C ABI of libyl_attention.so beyond its C++ interface.
 *
 * libyl_attention.so holds flashinfer's paged attention kernels (third-party,
 * compiled from the headers flashinfer ships) for the C++ Attention layer
 * (yllang::Attention, csrc/torch/attention.cpp), which plans each step into a
 * workspace it allocates.  This header adds one entry point for callers that
 * must not allocate device memory at all.
 */
#ifndef YL_ATTENTION_H_
#define YL_ATTENTION_H_

#include "yl_kvpath.h" /* yl_status, YL_API, cudaStream_t */

#ifdef __cplusplus
extern "C" {
#endif

#define YL_ATTN_BF16 0
#define YL_ATTN_FP16 1

/* Largest batch yl_paged_decode_attention_noalloc takes (its fixed scratch). */
#define YL_DECODE_NOALLOC_MAX_BATCH 16384

/*
 * Paged decode attention, one query row per sequence, that allocates nothing
 * (no counterpart in the reference: the reference's Attention::Forward is a
 * placeholder, src/include/layers/attention.h:55).
 *
 * Who needs it: a caller that cannot call cudaMalloc on its hot path — an
 * engine that reserves all device memory when it starts and hands nothing
 * out afterwards, or host code that runs under another framework's caching
 * allocator it has no handle on, where a raw allocation can fail for lack of
 * memory the cache holds or block until the device is idle.  The workspace
 * the planned path of yllang::Attention needs (split-KV partial outputs and
 * the plan's work lists) is replaced by a fixed array inside this library:
 * every sequence is one unit of work (no split of long sequences), and the
 * work lists live in a file-scope device array of
 * 2 * YL_DECODE_NOALLOC_MAX_BATCH + 64 int32 (about 128 KB) that every GPU
 * loading the library holds until the process exits.
 *
 * The first call on a device looks up that array's device address (once per
 * device, with the device current); make that first call before any stream
 * capture.  Every call rewrites the work lists for its batch, so a call
 * never depends on the previous call's contents, but all calls share the one
 * array: calls that overlap on the GPU (on different streams, without an
 * ordering between them) race on it.
 *
 * Semantics are those of the planned decode path: for each sequence i and
 * query head h, o[i, h] = softmax(q[i, h] . K_i^T * sm_scale) V_i over the
 * sequence's kv length (kv_indptr[i+1] - kv_indptr[i] - 1) * page_size +
 * kv_last_page_len[i], query heads mapped to KV heads in groups of
 * num_qo_heads / num_kv_heads (1, 2, 3, 4 or 8).  Pointers are device
 * pointers; strides are in elements.  o is written contiguously as
 * [batch_size, num_qo_heads, head_dim].  A batch of 0 is a no-op; a batch
 * above YL_DECODE_NOALLOC_MAX_BATCH returns YL_ERR_BAD_SIZE before any launch.
 */
typedef struct yl_decode_attention_args {
  const void *q;                    /* [batch, num_qo_heads, head_dim] rows                 */
  void *o;                          /* [batch, num_qo_heads, head_dim], contiguous          */
  const void *k_cache;              /* one layer's K pool, NHD [pages, page_size, Hk, D]    */
  const void *v_cache;              /* one layer's V pool, same strides                     */
  const int32_t *kv_indptr;         /* [batch + 1]                                          */
  const int32_t *kv_indices;        /* [kv_indptr[batch]] page ids                          */
  const int32_t *kv_last_page_len;  /* [batch]                                              */
  int64_t q_row_stride;             /* elements between query rows                          */
  int64_t q_head_stride;            /* elements between heads of a query row                */
  int64_t page_stride;              /* elements between pages of the pool                   */
  int64_t slot_stride;              /* elements between slots of a page                     */
  int64_t head_stride;              /* elements between heads of a slot                     */
  int32_t batch_size;               /* 0 .. YL_DECODE_NOALLOC_MAX_BATCH                     */
  int32_t num_qo_heads;
  int32_t num_kv_heads;
  int32_t head_dim;                 /* 64, 128 or 256                                       */
  int32_t page_size;
  int32_t dtype;                    /* YL_ATTN_BF16 or YL_ATTN_FP16 (q, pool and o)         */
  float sm_scale;                   /* usually 1 / sqrt(head_dim)                           */
} yl_decode_attention_args;

YL_API int yl_paged_decode_attention_noalloc(const yl_decode_attention_args *args, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* YL_ATTENTION_H_ */
