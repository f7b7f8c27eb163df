// yl_paged_decode_attention_noalloc (include/yl_attention.h): flashinfer's
// paged batch decode with its work lists in a fixed device array of this
// file instead of a caller's workspace, for callers that cannot allocate.
//
// The kernel reads, per CTA, the sequence it serves and the tile of that
// sequence (request_indices, kv_tile_indices) and the split size; the planned
// path fills those from a host plan into an allocated workspace and may split
// long sequences over CTAs (partial outputs in a float workspace).  Here every
// sequence is one unit: a small kernel writes request i = i, tile 0 for the
// call's batch into the array below, then the decode kernel runs without a
// split, so it needs no partial-output buffer.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <exception>
#include <flashinfer/attention/decode.cuh>
#include <flashinfer/attention/default_decode_params.cuh>
#include <flashinfer/attention/variants.cuh>
#include <mutex>
#include <vector>

#include "yl_attention.h"

namespace {

constexpr int kMax = YL_DECODE_NOALLOC_MAX_BATCH;
constexpr int kListWords = 2 * kMax + 64;  // request indices, tile indices, the split size, padding

// The work lists of the last call, shared by every call on this device.
static __device__ __align__(256) int32_t g_decode_lists[kListWords];

using Variant = flashinfer::DefaultAttention<false, false, false, false>;

// request i -> sequence i, tile 0 (no split); the split size word is read by
// the kernel but unused without a split, written 0.
__global__ void fill_decode_lists(int32_t batch) {
  const int32_t i = static_cast<int32_t>(blockIdx.x * blockDim.x + threadIdx.x);
  if (i < batch) {
    g_decode_lists[i] = i;
    g_decode_lists[kMax + i] = 0;
  }
  if (i == 0) g_decode_lists[2 * kMax] = 0;
}

// Device address of g_decode_lists on the current device, looked up once per
// device (a host-side use of the array's name is not a device address).
int lists_on_device(int32_t **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return YL_ERR_CUDA;
  }
  static std::mutex mu;
  static std::vector<int32_t *> addr;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(addr.size()) <= dev) addr.resize(dev + 1, nullptr);
  if (addr[dev] == nullptr) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_lists) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return YL_ERR_CUDA;
    }
    addr[dev] = static_cast<int32_t *>(p);
  }
  *out = addr[dev];
  return YL_OK;
}

template <typename T, uint32_t D>
int run(const yl_decode_attention_args &a, int32_t *lists, cudaStream_t stream) {
  using Params = flashinfer::BatchDecodeParams<T, T, T, int32_t>;
  const int64_t strides[3] = {a.page_stride, a.slot_stride, a.head_stride};
  Params p;
  p.q = static_cast<T *>(const_cast<void *>(a.q));
  p.paged_kv = flashinfer::paged_kv_t<T, int32_t>(
      static_cast<uint32_t>(a.num_kv_heads), static_cast<uint32_t>(a.page_size), D,
      static_cast<uint32_t>(a.batch_size), flashinfer::QKVLayout::kNHD, static_cast<T *>(const_cast<void *>(a.k_cache)),
      static_cast<T *>(const_cast<void *>(a.v_cache)), strides, const_cast<int32_t *>(a.kv_indices),
      const_cast<int32_t *>(a.kv_indptr), const_cast<int32_t *>(a.kv_last_page_len));
  p.o = static_cast<T *>(a.o);
  p.lse = nullptr;
  p.num_qo_heads = static_cast<uint32_t>(a.num_qo_heads);
  p.q_stride_n = static_cast<int32_t>(a.q_row_stride);
  p.q_stride_h = static_cast<int32_t>(a.q_head_stride);
  p.window_left = -1;
  p.logits_soft_cap = 0.f;
  p.sm_scale = a.sm_scale;
  p.rope_rcp_scale = 1.f;
  p.rope_rcp_theta = 1.f;
  p.request_indices = lists;
  p.kv_tile_indices = lists + kMax;
  p.kv_chunk_size_ptr = lists + 2 * kMax;
  p.o_indptr = nullptr;
  p.block_valid_mask = nullptr;
  p.padded_batch_size = static_cast<uint32_t>(a.batch_size);
  p.partition_kv = false;
  const cudaError_t e = flashinfer::BatchDecodeWithPagedKVCacheDispatched<D, flashinfer::PosEncodingMode::kNone,
                                                                          Variant>(p, nullptr, nullptr, false, stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return YL_ERR_CUDA;
  }
  return YL_OK;
}

template <typename T>
int by_dim(const yl_decode_attention_args &a, int32_t *lists, cudaStream_t stream) {
  switch (a.head_dim) {
    case 64: return run<T, 64>(a, lists, stream);
    case 128: return run<T, 128>(a, lists, stream);
    default: return run<T, 256>(a, lists, stream);
  }
}

}  // namespace

extern "C" int yl_paged_decode_attention_noalloc(const yl_decode_attention_args *a, cudaStream_t stream) {
  if (a == nullptr) return YL_ERR_NULL_ARG;
  if (a->batch_size < 0 || a->batch_size > kMax) return YL_ERR_BAD_SIZE;
  if (a->batch_size == 0) return YL_OK;
  if (!a->q || !a->o || !a->k_cache || !a->v_cache || !a->kv_indptr || !a->kv_indices || !a->kv_last_page_len)
    return YL_ERR_NULL_ARG;
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256) return YL_ERR_UNSUPPORTED;
  if (a->dtype != YL_ATTN_BF16 && a->dtype != YL_ATTN_FP16) return YL_ERR_UNSUPPORTED;
  if (a->page_size < 1 || a->num_kv_heads < 1 || a->num_qo_heads < a->num_kv_heads ||
      a->num_qo_heads % a->num_kv_heads != 0)
    return YL_ERR_BAD_SIZE;
  const int group = a->num_qo_heads / a->num_kv_heads;
  if (group != 1 && group != 2 && group != 3 && group != 4 && group != 8) return YL_ERR_UNSUPPORTED;
  int32_t *lists = nullptr;
  int rc = lists_on_device(&lists);
  if (rc != YL_OK) return rc;
  fill_decode_lists<<<(a->batch_size + 255) / 256, 256, 0, stream>>>(a->batch_size);
  if (cudaGetLastError() != cudaSuccess) return YL_ERR_CUDA;
  try {
    rc = a->dtype == YL_ATTN_FP16 ? by_dim<__half>(*a, lists, stream) : by_dim<__nv_bfloat16>(*a, lists, stream);
  } catch (const std::exception &) {
    rc = YL_ERR_UNSUPPORTED;
  }
  return rc;
}
