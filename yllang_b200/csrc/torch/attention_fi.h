// Torch-free bridge from yllang::Attention to flashinfer's paged attention
// kernels: batch decode over a paged K/V pool, and causal batch prefill over
// it.  flashinfer is the third-party consumer of the index arrays this library
// builds (kv_indptr, kv_indices, kv_last_page_len, qo_indptr); its kernels are
// compiled here, unchanged, from the headers flashinfer ships.
//
// Every entry returns an empty string on success, else the error message
// (flashinfer's or the CUDA runtime's); no exception leaves this interface.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

// The library is built with hidden visibility; these are its exports.
#define YL_FI_API __attribute__((visibility("default")))

namespace yllang {
namespace fi {

enum class DType { kBF16, kFP16 };

// Scratch the planner and the kernels share: a device float buffer (split-KV
// partial outputs), a device int buffer and a page-locked host int buffer of
// the same size (the plan's request/tile lists, staged on the host and copied
// over on the plan's stream).
struct Workspace {
  void *float_buffer;
  size_t float_bytes;
  void *int_buffer;
  void *int_host_buffer;
  size_t int_bytes;
};

struct Shape {
  int batch;         // sequences
  int num_qo_heads;  // query heads on this GPU
  int num_kv_heads;  // K/V heads on this GPU (num_qo_heads % num_kv_heads == 0)
  int head_dim;      // 64, 128 or 256
  int page_size;
  DType dtype;       // q, the pool and the output share it
};

// One layer's paged pool, NHD: page p, in-page slot n, head h, element d at
// base + p * stride_page + n * stride_n + h * stride_h + d (element strides).
struct PagedPool {
  void *k;
  void *v;
  int64_t stride_page;
  int64_t stride_n;
  int64_t stride_h;
  int32_t *kv_indptr;         // [batch + 1] device
  int32_t *kv_indices;        // [kv_indptr[batch]] device
  int32_t *kv_last_page_len;  // [batch] device
};

// Queries (and the output, same strides): row t, head h at base + t * stride_n + h * stride_h.
struct Rows {
  const void *q;
  void *o;
  int64_t stride_n;
  int64_t stride_h;
  int64_t o_stride_n;
  int64_t o_stride_h;
};

// Decode: one query row per sequence.  kv_indptr_host is the step's
// kv_indptr on the host (the planner splits long sequences over CTAs).
YL_FI_API std::string PlanDecode(const Workspace &ws, const Shape &s, const int32_t *kv_indptr_host, cudaStream_t stream,
                       std::vector<int64_t> *plan);
YL_FI_API std::string RunDecode(const Workspace &ws, const Shape &s, const std::vector<int64_t> &plan, const Rows &rows,
                      const PagedPool &pool, float sm_scale, cudaStream_t stream);

// Prefill: qo_indptr rows per sequence, query row t of sequence i at position
// (kv length of i) - (new rows of i) + t, attending causally.
YL_FI_API std::string PlanPrefill(const Workspace &ws, const Shape &s, const int32_t *qo_indptr_host,
                        const int32_t *kv_indptr_host, cudaStream_t stream, std::vector<int64_t> *plan);
YL_FI_API std::string RunPrefill(const Workspace &ws, const Shape &s, const std::vector<int64_t> &plan, const Rows &rows,
                       int32_t *qo_indptr_device, const PagedPool &pool, float sm_scale, cudaStream_t stream);

}  // namespace fi
}  // namespace yllang
