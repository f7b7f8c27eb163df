// Range expansion for sm_100a: the flat page-table indices NextBatch builds
// with Make2DIndices (src/include/batch/batch_manager.h:30-51), where the host
// assigns them one libtorch scalar at a time (batch_manager.h:45-47).
//
// Every block scans the range lengths itself, 512 ranges at a time, into
// shared-memory offsets; the output positions of each chunk are cut into
// tiles of 512, dealt to the grid's warps in turn.  A lane finds the range of
// its first position by a binary search over the chunk's offsets, then walks
// forward through its 16 positions (32 apart, so each store instruction of
// the warp writes 256 contiguous bytes).  A range costs 24 bytes of reads per
// block, an index 8 bytes of writes: at the batch sizes NextBatch sees
// (ranges in the hundreds or thousands, indices in the hundreds of thousands)
// the kernel is bound by its int64 stores.
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

#include "common.cuh"

namespace ylk {

constexpr int kRangeThreads = 512;            // ranges per scan chunk (one per thread)
constexpr int64_t kRangeLenCap = 1ll << 40;   // longer ranges count as this long
constexpr int64_t kMaxRanges = 1ll << 22;     // so that sums of capped lengths stay below 2^62
constexpr int kWarpTile = 32 * 16;            // output positions a warp writes per tile (16 per lane)

struct RangesParams {
  const int64_t *ranges;
  int64_t *indices;
  int64_t *count;
  uint32_t *error_word;
  int64_t capacity;
  int32_t num_ranges;
};

__device__ __forceinline__ int64_t warp_inclusive_scan(int64_t x, int lane) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  return x;
}

__global__ void __launch_bounds__(kRangeThreads) make_2d_indices_kernel(const __grid_constant__ RangesParams p) {
  __shared__ int64_t off[kRangeThreads + 1];          // chunk-relative offsets; off[n] = the chunk's total
  __shared__ int64_t first[kRangeThreads];            // first index of each range of the chunk
  __shared__ int64_t warp_base[kRangeThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool report = blockIdx.x == 0;  // every block sees the same ranges: one reports
  const int64_t gwarp = static_cast<int64_t>(blockIdx.x) * (kRangeThreads / 32) + warp;
  const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * (kRangeThreads / 32) * kWarpTile;
  int64_t carry = 0;  // indices of the chunks before this one
  pdl_wait();  // the ranges may be written by the kernel just before this one
  for (int c0 = 0; c0 < p.num_ranges; c0 += kRangeThreads) {
    const int n = min(kRangeThreads, p.num_ranges - c0);
    int64_t len = 0, start = 0;
    if (tid < n) {
      const int64_t *r = p.ranges + 3ll * (c0 + tid);
      const int64_t row = __ldg(r), lo = __ldg(r + 1), hi = __ldg(r + 2);
      if (row < 0 || lo < 0 || hi < lo) {
        if (report) raise_deverr(p.error_word, YL_DEVERR_NEGATIVE_LEN);
      } else if (row > LLONG_MAX - hi) {
        if (report) raise_deverr(p.error_word, YL_DEVERR_INDEX_RANGE);
      } else {
        len = min(hi - lo, kRangeLenCap);
        start = row + lo;
      }
    }
    const int64_t x = warp_inclusive_scan(len, lane);
    if (lane == 31) warp_base[warp] = x;
    __syncthreads();
    if (warp == 0) {
      const int64_t w = lane < kRangeThreads / 32 ? warp_base[lane] : 0;
      const int64_t s = warp_inclusive_scan(w, lane);  // every lane has read warp_base before any writes it
      if (lane < kRangeThreads / 32) warp_base[lane] = s - w;
    }
    __syncthreads();
    off[tid + 1] = x + warp_base[warp];
    first[tid] = start;
    if (tid == 0) off[0] = 0;
    __syncthreads();
    const int64_t total = off[n];
    const int64_t limit = min(total, p.capacity - carry);  // <= 0 once the output is full
    int64_t *out = p.indices + carry;
    for (int64_t t0 = gwarp * kWarpTile; t0 < limit; t0 += warp_stride) {
      int64_t q = t0 + lane;
      if (q >= limit) continue;
      // The last range k < n with off[k] <= q: off[k + 1] > q, so range k is
      // not empty and holds position q.  Later positions of the lane walk
      // forward from there (a range change is rare: ranges are long).
      int k = 0;
#pragma unroll
      for (int step = kRangeThreads / 2; step > 0; step >>= 1)
        if (k + step < n && off[k + step] <= q) k += step;
      int64_t next = off[k + 1];
      int64_t base = first[k] - off[k];
      const int64_t end = min(t0 + kWarpTile, limit);
      for (; q < end; q += 32) {
        while (q >= next) {  // ends: q < limit <= off[n]
          ++k;
          next = off[k + 1];
          base = first[k] - off[k];
        }
        out[q] = base + q;
      }
    }
    carry += total;
    __syncthreads();  // off / first / warp_base are rewritten by the next chunk
  }
  if (report && tid == 0) {
    if (carry > p.capacity) raise_deverr(p.error_word, YL_DEVERR_INDICES_CAP);
    if (p.count != nullptr) *p.count = carry;
  }
}

}  // namespace ylk

extern "C" int yl_make_2d_indices(const yl_ranges_args *a, cudaStream_t stream) {
  using namespace ylk;
  clear_last_error();
  if (a == nullptr) return fail(YL_ERR_NULL_ARG, "yl_make_2d_indices: args is NULL");
  if (a->num_ranges < 0) return fail(YL_ERR_BAD_SIZE, "yl_make_2d_indices: num_ranges=%lld < 0", a->num_ranges);
  if (a->indices_capacity < 0)
    return fail(YL_ERR_BAD_SIZE, "yl_make_2d_indices: indices_capacity=%lld < 0", a->indices_capacity);
  if (a->num_ranges > kMaxRanges)
    return fail(YL_ERR_UNSUPPORTED, "yl_make_2d_indices: num_ranges=%lld exceeds %lld", a->num_ranges, kMaxRanges);
  if (a->indices_capacity >= kRangeLenCap)
    return fail(YL_ERR_UNSUPPORTED, "yl_make_2d_indices: indices_capacity=%lld is not below 2^40",
                a->indices_capacity);
  if (a->num_ranges == 0 && a->count == nullptr) return YL_OK;
  if (a->num_ranges > 0 && a->ranges == nullptr) return fail(YL_ERR_NULL_ARG, "yl_make_2d_indices: ranges is NULL");
  if (a->indices_capacity > 0 && a->indices == nullptr)
    return fail(YL_ERR_NULL_ARG, "yl_make_2d_indices: indices is NULL");
  const uintptr_t bits = reinterpret_cast<uintptr_t>(a->ranges) | reinterpret_cast<uintptr_t>(a->indices) |
                         reinterpret_cast<uintptr_t>(a->count);
  if ((bits & 7u) != 0) return fail(YL_ERR_ALIGNMENT, "yl_make_2d_indices: ranges, indices and count must be 8-byte aligned");

  RangesParams p;
  p.ranges = a->ranges;
  p.indices = a->indices;
  p.count = a->count;
  p.error_word = a->error_word;
  p.capacity = a->indices_capacity;
  p.num_ranges = static_cast<int32_t>(a->num_ranges);
  // One tile per warp over the output; at most two blocks per SM, each of
  // which rescans every range.
  const int64_t per_block = static_cast<int64_t>(kRangeThreads / 32) * kWarpTile;
  const int64_t want = (a->indices_capacity + per_block - 1) / per_block;
  const int64_t cap = 2ll * sm_count();
  const unsigned grid = static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
  return launch_dependent(make_2d_indices_kernel, dim3(grid), dim3(kRangeThreads), 0, stream,
                          "yl_make_2d_indices launch", p);
}
