// Parity harness: the reference's own StoreKVCache launcher and kernel
// (src/kvcache/store_kv_cache.cu:46-163), compiled from the reference source
// tree in place by oracle/Makefile, behind a C entry point that takes raw
// device pointers.  TEST INFRASTRUCTURE ONLY.
//
// The reference instantiates its launcher for one row size, kElementSize
// (store_kv_cache.cu:165, src/include/config/config.h:19); here it is
// instantiated for the four row sizes its Copy<> accepts (512..4096 bytes;
// 256-byte rows fail its static_assert, src/include/cuda/memory.cuh:151).
// The launcher always reads int64 indices (store_kv_cache.cu:127), so callers
// pass int64 slots.
#include "kvcache/store_kv_cache.cu"

namespace yllang {
template auto StoreKVCache<512>(const torch::Tensor &, const torch::Tensor &, const torch::Tensor &,
                                const torch::Tensor &, const torch::Tensor &) -> void;
template auto StoreKVCache<1024>(const torch::Tensor &, const torch::Tensor &, const torch::Tensor &,
                                 const torch::Tensor &, const torch::Tensor &) -> void;
template auto StoreKVCache<4096>(const torch::Tensor &, const torch::Tensor &, const torch::Tensor &,
                                 const torch::Tensor &, const torch::Tensor &) -> void;
}  // namespace yllang

namespace {
torch::Dtype dtype_of(int code) {
  switch (code) {
    case 0: return torch::kBFloat16;
    case 1: return torch::kFloat16;
    case 2: return torch::kFloat32;
    default: return torch::kUInt8;
  }
}
}  // namespace

// k, v:       [n, row_elems] with row stride k_stride_elems (elements)
// caches:     [cache_rows, row_elems] with row stride cache_stride_elems
// indices:    int64 [n]
// dtype_code: 0 bf16, 1 fp16, 2 fp32.
// Returns 0, -1 for an unsupported row size, -2 if the launcher threw.
extern "C" int ref_store_kv_cache(int64_t row_bytes, int dtype_code, int device, void *k, void *v, void *k_cache,
                                  void *v_cache, const int64_t *indices, int64_t n, int64_t k_stride_elems,
                                  int64_t cache_rows, int64_t cache_stride_elems) {
  try {
    const auto dt = dtype_of(dtype_code);
    const auto opt = torch::TensorOptions().dtype(dt).device(torch::kCUDA, device);
    const int64_t item = torch::elementSize(dt);
    const int64_t e = row_bytes / item;
    auto tk = torch::from_blob(k, {n, e}, {k_stride_elems, 1}, opt);
    auto tv = torch::from_blob(v, {n, e}, {k_stride_elems, 1}, opt);
    auto tkc = torch::from_blob(k_cache, {cache_rows, e}, {cache_stride_elems, 1}, opt);
    auto tvc = torch::from_blob(v_cache, {cache_rows, e}, {cache_stride_elems, 1}, opt);
    auto ti = torch::from_blob(const_cast<int64_t *>(indices), {n}, {1},
                               torch::TensorOptions().dtype(torch::kInt64).device(torch::kCUDA, device));
    switch (row_bytes) {
      case 512: yllang::StoreKVCache<512>(tk, tv, tkc, tvc, ti); break;
      case 1024: yllang::StoreKVCache<1024>(tk, tv, tkc, tvc, ti); break;
      case 2048: yllang::StoreKVCache<2048>(tk, tv, tkc, tvc, ti); break;
      case 4096: yllang::StoreKVCache<4096>(tk, tv, tkc, tvc, ti); break;
      default: return -1;
    }
  } catch (const std::exception &) {
    return -2;
  }
  return 0;
}
