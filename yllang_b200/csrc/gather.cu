// Row gather for sm_100a: out[i] <- table[indices[i]] (the embedding lookup),
// on the same copy engine as the KV store.
//
// Reference behaviour (src/layers/index.cu:49-77): one warp per output row,
// 16-byte copies.  Here lane groups of G lanes copy a row as G x VPL vectors
// of W bytes (the store's row shapes); a group takes R rows per iteration,
// loads their R indices, then issues every row load before any store.  An
// index outside the table zero-fills its output row.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "common.cuh"
#include "store_device.cuh"

namespace ylk {

struct GatherParams {
  const char *table;
  char *out;
  const void *indices;
  int64_t table_row_stride;
  int64_t out_row_stride;
  int64_t num_rows;
  uint32_t *error_word;
  uint32_t n;
  uint32_t row_units;
};

template <typename IdxT>
__device__ __forceinline__ int64_t load_index(const void *p, uint32_t i) {
  return static_cast<int64_t>(__ldg(static_cast<const IdxT *>(p) + i));
}

// True when the index names a table row; -1 is skipped silently, anything
// else out of range is skipped and reported.
__device__ __forceinline__ bool index_ok(int64_t r, const GatherParams &p) {
  if (r >= 0 && (p.num_rows <= 0 || r < p.num_rows)) return true;
  if (r != -1) raise_deverr(p.error_word, YL_DEVERR_INDEX_RANGE);
  return false;
}

template <int W, int G, int VPL, int R, typename IdxT>
__global__ void __launch_bounds__(256) gather_rows_kernel(const __grid_constant__ GatherParams p) {
  const uint32_t lane = threadIdx.x % G;
  const uint32_t group = (blockIdx.x * blockDim.x + threadIdx.x) / G;
  const uint32_t num_groups = (gridDim.x * blockDim.x) / G;
  pdl_wait();  // the indices may be written by the kernel just before this one
  for (uint32_t base = group * R; base < p.n; base += num_groups * R) {
    int64_t src[R];
#pragma unroll
    for (int r = 0; r < R; ++r) src[r] = base + r < p.n ? load_index<IdxT>(p.indices, base + r) : -1;
    Vec<W> data[R][VPL];
    bool ok[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      ok[r] = base + r < p.n && index_ok(src[r], p);
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        if (ok[r]) {
          load_vec(data[r][j], p.table + src[r] * p.table_row_stride + (j * G + lane) * W);
        } else {
#pragma unroll
          for (int q = 0; q < W / 4; ++q) data[r][j].r[q] = 0u;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (base + r < p.n) {
        char *dst = p.out + static_cast<int64_t>(base + r) * p.out_row_stride;
#pragma unroll
        for (int j = 0; j < VPL; ++j) store_vec(dst + (j * G + lane) * W, data[r][j]);
      }
    }
  }
}

// Any row size and alignment: unit U, one warp per row.
template <typename U, typename IdxT>
__global__ void __launch_bounds__(256) gather_rows_generic_kernel(const __grid_constant__ GatherParams p) {
  const uint32_t lane = threadIdx.x % 32;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const uint32_t num_warps = (gridDim.x * blockDim.x) / 32;
  pdl_wait();
  for (uint32_t row = warp; row < p.n; row += num_warps) {
    const int64_t s = load_index<IdxT>(p.indices, row);
    U *dst = reinterpret_cast<U *>(p.out + static_cast<int64_t>(row) * p.out_row_stride);
    if (index_ok(s, p)) {
      const U *src = reinterpret_cast<const U *>(p.table + s * p.table_row_stride);
      for (uint32_t u = lane; u < p.row_units; u += 32) dst[u] = src[u];
    } else {
      for (uint32_t u = lane; u < p.row_units; u += 32) dst[u] = U{};
    }
  }
}

int blocks_per_sm(const void *fn, size_t smem);  // kv_store.cu, at 256 threads

}  // namespace ylk

extern "C" int yl_gather_rows(const yl_gather_args *a, cudaStream_t stream) {
  using namespace ylk;
  clear_last_error();
  if (a == nullptr) return fail(YL_ERR_NULL_ARG, "yl_gather_rows: args is NULL");
  if (a->num_indices < 0) return fail(YL_ERR_BAD_SIZE, "yl_gather_rows: num_indices=%lld < 0", a->num_indices);
  if (a->row_bytes <= 0) return fail(YL_ERR_BAD_SIZE, "yl_gather_rows: row_bytes=%lld <= 0", a->row_bytes);
  if (a->reserved != 0) return fail(YL_ERR_BAD_SIZE, "yl_gather_rows: reserved=%lld must be 0", a->reserved);
  if (a->index_is_int64 != 0 && a->index_is_int64 != 1)
    return fail(YL_ERR_BAD_SIZE, "yl_gather_rows: index_is_int64=%lld must be 0 or 1", a->index_is_int64);
  if (a->num_indices == 0) return YL_OK;
  if (!a->table || !a->out || !a->indices)
    return fail(YL_ERR_NULL_ARG, "yl_gather_rows: table, out and indices must be non-NULL");
  if (a->table_row_stride < a->row_bytes || a->out_row_stride < a->row_bytes)
    return fail(YL_ERR_BAD_SIZE, "yl_gather_rows: row strides must be >= row_bytes=%lld", a->row_bytes);
  if (a->num_indices >= (1ll << 31))
    return fail(YL_ERR_UNSUPPORTED, "yl_gather_rows: num_indices=%lld exceeds 2^31-1", a->num_indices);
  const size_t ib = a->index_is_int64 ? 8 : 4;
  if ((reinterpret_cast<uintptr_t>(a->indices) & (ib - 1)) != 0)
    return fail(YL_ERR_ALIGNMENT, "yl_gather_rows: indices pointer is not %lld-byte aligned", (long long)ib);
  const uintptr_t bits = reinterpret_cast<uintptr_t>(a->table) | reinterpret_cast<uintptr_t>(a->out) |
                         static_cast<uintptr_t>(a->row_bytes) | static_cast<uintptr_t>(a->table_row_stride) |
                         static_cast<uintptr_t>(a->out_row_stride);
  int unit = 16;
  while (unit > 1 && (bits & static_cast<uintptr_t>(unit - 1)) != 0) unit >>= 1;
  if (a->row_bytes / unit >= (1ll << 31))
    return fail(YL_ERR_UNSUPPORTED, "yl_gather_rows: row_bytes=%lld too large", a->row_bytes);

  GatherParams p;
  p.table = static_cast<const char *>(a->table);
  p.out = static_cast<char *>(a->out);
  p.indices = a->indices;
  p.table_row_stride = a->table_row_stride;
  p.out_row_stride = a->out_row_stride;
  p.num_rows = a->num_rows;
  p.error_word = a->error_word;
  p.n = static_cast<uint32_t>(a->num_indices);
  p.row_units = static_cast<uint32_t>(a->row_bytes / unit);

  using Kernel = void (*)(GatherParams);
  Kernel fn = nullptr;
  int group = 32, rows = 1;
  const bool i64 = a->index_is_int64 != 0;
  auto pick = [&](auto shape) {
    using S = decltype(shape);
    fn = i64 ? gather_rows_kernel<S::W, S::G, S::VPL, S::R, int64_t> : gather_rows_kernel<S::W, S::G, S::VPL, S::R, int32_t>;
    group = S::G;
    rows = S::R;
  };
  bool fast = false;
  if (unit == 16 && fast_vector_bytes() == 32 && (bits & 31u) == 0) fast = dispatch_row_shape(a->row_bytes, 32, pick);
  if (!fast && unit == 16) fast = dispatch_row_shape(a->row_bytes, 16, pick);
  if (!fast) {
    switch (unit) {
      case 16: fn = i64 ? gather_rows_generic_kernel<uint4, int64_t> : gather_rows_generic_kernel<uint4, int32_t>; break;
      case 8: fn = i64 ? gather_rows_generic_kernel<uint2, int64_t> : gather_rows_generic_kernel<uint2, int32_t>; break;
      case 4: fn = i64 ? gather_rows_generic_kernel<uint32_t, int64_t> : gather_rows_generic_kernel<uint32_t, int32_t>; break;
      case 2: fn = i64 ? gather_rows_generic_kernel<uint16_t, int64_t> : gather_rows_generic_kernel<uint16_t, int32_t>; break;
      default: fn = i64 ? gather_rows_generic_kernel<uint8_t, int64_t> : gather_rows_generic_kernel<uint8_t, int32_t>; break;
    }
    group = 32;
    rows = 1;
  }
  const uint64_t rows_per_block = static_cast<uint64_t>(256 / group) * rows;
  const uint64_t want = (static_cast<uint64_t>(p.n) + rows_per_block - 1) / rows_per_block;
  const uint64_t cap = static_cast<uint64_t>(sm_count()) * blocks_per_sm(reinterpret_cast<const void *>(fn), 0);
  return launch_dependent(fn, dim3(static_cast<unsigned>(want < cap ? want : cap)), dim3(256), 0, stream,
                          "yl_gather_rows launch", p);
}
