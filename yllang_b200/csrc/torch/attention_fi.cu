// flashinfer's paged decode and causal paged prefill, instantiated for the
// pools this library stores into (bf16 / fp16, head_dim 64 / 128 / 256, NHD),
// behind the torch-free interface of attention_fi.h.  Planning and launching
// follow flashinfer's own host flow: a plan pass that sizes the work split
// from the host indptr arrays, then the kernel launch with the plan's lists.
#include "attention_fi.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <exception>
#include <flashinfer/attention/decode.cuh>
#include <flashinfer/attention/default_decode_params.cuh>
#include <flashinfer/attention/default_prefill_params.cuh>
#include <flashinfer/attention/prefill.cuh>
#include <flashinfer/attention/scheduler.cuh>
#include <flashinfer/attention/variants.cuh>

namespace yllang {
namespace fi {
namespace {

using flashinfer::DecodePlanInfo;
using flashinfer::MaskMode;
using flashinfer::PosEncodingMode;
using flashinfer::PrefillPlanInfo;
using flashinfer::QKVLayout;
using Variant = flashinfer::DefaultAttention</*custom mask*/ false, /*sliding window*/ false,
                                             /*soft cap*/ false, /*alibi*/ false>;

template <typename T>
T *at(void *base, int64_t offset) {
  return reinterpret_cast<T *>(static_cast<char *>(base) + offset);
}

std::string cuda_error(const char *what, cudaError_t e) {
  return std::string(what) + ": " + cudaGetErrorString(e);
}

// Calls f(T{}, std::integral_constant<int, D>{}) for the shape's element type
// and head dim; returns an error message for anything else.
template <typename F>
std::string dispatch(const Shape &s, F &&f) {
  auto by_dim = [&](auto t) -> std::string {
    switch (s.head_dim) {
      case 64: return f(t, std::integral_constant<int, 64>{});
      case 128: return f(t, std::integral_constant<int, 128>{});
      case 256: return f(t, std::integral_constant<int, 256>{});
      default: return "attention: head_dim " + std::to_string(s.head_dim) + " (64, 128 or 256 supported)";
    }
  };
  if (s.dtype == DType::kBF16) return by_dim(__nv_bfloat16{});
  return by_dim(__half{});
}

template <typename T>
flashinfer::paged_kv_t<T, int32_t> paged(const Shape &s, const PagedPool &pool) {
  const int64_t strides[3] = {pool.stride_page, pool.stride_n, pool.stride_h};
  return flashinfer::paged_kv_t<T, int32_t>(static_cast<uint32_t>(s.num_kv_heads), static_cast<uint32_t>(s.page_size),
                                            static_cast<uint32_t>(s.head_dim), static_cast<uint32_t>(s.batch),
                                            QKVLayout::kNHD, static_cast<T *>(pool.k), static_cast<T *>(pool.v),
                                            strides, pool.kv_indices, pool.kv_indptr, pool.kv_last_page_len);
}

// flashinfer reports bad shapes by throwing; keep exceptions inside.
template <typename F>
std::string guarded(F &&f) {
  try {
    return f();
  } catch (const std::exception &e) {
    return std::string("flashinfer: ") + e.what();
  }
}

}  // namespace

std::string PlanDecode(const Workspace &ws, const Shape &s, const int32_t *kv_indptr_host, cudaStream_t stream,
                       std::vector<int64_t> *plan) {
  return guarded([&] {
    return dispatch(s, [&](auto t, auto dim) -> std::string {
      using T = decltype(t);
      constexpr uint32_t D = decltype(dim)::value;
      using Params = flashinfer::BatchDecodeParams<T, T, T, int32_t>;
      DecodePlanInfo info;
      cudaError_t e = cudaSuccess;
      DISPATCH_GQA_GROUP_SIZE(s.num_qo_heads / s.num_kv_heads, GROUP_SIZE, {
        auto estimate = flashinfer::BatchDecodeWithPagedKVCacheWorkEstimationDispatched<
            GROUP_SIZE, D, PosEncodingMode::kNone, Variant, Params>;
        e = flashinfer::DecodePlan<D, PosEncodingMode::kNone, Variant, Params>(
            ws.float_buffer, ws.float_bytes, ws.int_buffer, ws.int_host_buffer, ws.int_bytes, info,
            const_cast<int32_t *>(kv_indptr_host), static_cast<uint32_t>(s.batch),
            static_cast<uint32_t>(s.num_qo_heads), static_cast<uint32_t>(s.page_size),
            /*enable_cuda_graph=*/false, stream, estimate);
      });
      if (e != cudaSuccess) return cuda_error("attention decode plan", e);
      *plan = info.ToVector();
      return std::string();
    });
  });
}

std::string RunDecode(const Workspace &ws, const Shape &s, const std::vector<int64_t> &plan, const Rows &rows,
                      const PagedPool &pool, float sm_scale, cudaStream_t stream) {
  return guarded([&] {
    return dispatch(s, [&](auto t, auto dim) -> std::string {
      using T = decltype(t);
      constexpr uint32_t D = decltype(dim)::value;
      using Params = flashinfer::BatchDecodeParams<T, T, T, int32_t>;
      DecodePlanInfo info;
      info.FromVector(plan);
      if (rows.o_stride_n != static_cast<int64_t>(s.num_qo_heads) * D || rows.o_stride_h != D)
        return std::string("attention decode: the output must be contiguous [batch, heads, head_dim]");
      Params p;
      p.q = static_cast<T *>(const_cast<void *>(rows.q));
      p.paged_kv = paged<T>(s, pool);
      p.o = static_cast<T *>(rows.o);
      p.lse = nullptr;
      p.num_qo_heads = static_cast<uint32_t>(s.num_qo_heads);
      p.q_stride_n = static_cast<int32_t>(rows.stride_n);
      p.q_stride_h = static_cast<int32_t>(rows.stride_h);
      p.window_left = -1;
      p.logits_soft_cap = 0.f;
      p.sm_scale = sm_scale;
      p.rope_rcp_scale = 1.f;
      p.rope_rcp_theta = 1.f;
      p.request_indices = at<int32_t>(ws.int_buffer, info.request_indices_offset);
      p.kv_tile_indices = at<int32_t>(ws.int_buffer, info.kv_tile_indices_offset);
      p.o_indptr = at<int32_t>(ws.int_buffer, info.o_indptr_offset);
      p.kv_chunk_size_ptr = at<int32_t>(ws.int_buffer, info.kv_chunk_size_ptr_offset);
      p.block_valid_mask = nullptr;
      p.padded_batch_size = static_cast<uint32_t>(info.padded_batch_size);
      T *tmp_v = nullptr;
      float *tmp_s = nullptr;
      if (info.split_kv) {
        tmp_v = at<T>(ws.float_buffer, info.v_offset);
        tmp_s = at<float>(ws.float_buffer, info.s_offset);
      }
      const cudaError_t e = flashinfer::BatchDecodeWithPagedKVCacheDispatched<D, PosEncodingMode::kNone, Variant>(
          p, tmp_v, tmp_s, /*enable_pdl=*/false, stream);
      if (e != cudaSuccess) return cuda_error("attention decode", e);
      return std::string();
    });
  });
}

std::string PlanPrefill(const Workspace &ws, const Shape &s, const int32_t *qo_indptr_host,
                        const int32_t *kv_indptr_host, cudaStream_t stream, std::vector<int64_t> *plan) {
  return guarded([&]() -> std::string {
    PrefillPlanInfo info;
    const cudaError_t e = flashinfer::PrefillPlan<int32_t>(
        ws.float_buffer, ws.float_bytes, ws.int_buffer, ws.int_host_buffer, ws.int_bytes, info,
        const_cast<int32_t *>(qo_indptr_host), const_cast<int32_t *>(kv_indptr_host),
        static_cast<uint32_t>(qo_indptr_host[s.batch]), static_cast<uint32_t>(s.batch),
        static_cast<uint32_t>(s.num_qo_heads), static_cast<uint32_t>(s.num_kv_heads),
        static_cast<uint32_t>(s.head_dim), static_cast<uint32_t>(s.head_dim), static_cast<uint32_t>(s.page_size),
        /*enable_cuda_graph=*/false, /*sizeof_dtype_o=*/2, /*window_left=*/-1, /*fixed_split_size=*/-1,
        /*disable_split_kv=*/false, /*num_colocated_ctas=*/0, stream);
    if (e != cudaSuccess) return cuda_error("attention prefill plan", e);
    *plan = info.ToVector();
    return std::string();
  });
}

std::string RunPrefill(const Workspace &ws, const Shape &s, const std::vector<int64_t> &plan, const Rows &rows,
                       int32_t *qo_indptr_device, const PagedPool &pool, float sm_scale, cudaStream_t stream) {
  return guarded([&] {
    return dispatch(s, [&](auto t, auto dim) -> std::string {
      using T = decltype(t);
      constexpr uint32_t D = decltype(dim)::value;
      using Params = flashinfer::BatchPrefillPagedParams<T, T, T, int32_t>;
      PrefillPlanInfo info;
      info.FromVector(plan);
      if (rows.o_stride_n != static_cast<int64_t>(s.num_qo_heads) * D || rows.o_stride_h != D)
        return std::string("attention prefill: the output must be contiguous [rows, heads, head_dim]");
      Params p;
      p.q = static_cast<T *>(const_cast<void *>(rows.q));
      p.paged_kv = paged<T>(s, pool);
      p.q_indptr = qo_indptr_device;
      p.o = static_cast<T *>(rows.o);
      p.lse = nullptr;
      p.num_qo_heads = static_cast<uint32_t>(s.num_qo_heads);
      p.group_size = flashinfer::uint_fastdiv(static_cast<uint32_t>(s.num_qo_heads / s.num_kv_heads));
      p.q_stride_n = static_cast<int32_t>(rows.stride_n);
      p.q_stride_h = static_cast<int32_t>(rows.stride_h);
      p.window_left = -1;
      p.logits_soft_cap = 0.f;
      p.sm_scale = sm_scale;
      p.rope_rcp_scale = 1.f;
      p.rope_rcp_theta = 1.f;
      p.request_indices = at<int32_t>(ws.int_buffer, info.request_indices_offset);
      p.qo_tile_indices = at<int32_t>(ws.int_buffer, info.qo_tile_indices_offset);
      p.kv_tile_indices = at<int32_t>(ws.int_buffer, info.kv_tile_indices_offset);
      p.o_indptr = at<int32_t>(ws.int_buffer, info.o_indptr_offset);
      p.kv_chunk_size_ptr = at<int32_t>(ws.int_buffer, info.kv_chunk_size_ptr_offset);
      p.merge_indptr = nullptr;
      p.block_valid_mask = nullptr;
      p.total_num_rows = nullptr;
      p.padded_batch_size = static_cast<uint32_t>(info.padded_batch_size);
      p.max_total_num_rows = static_cast<uint32_t>(info.total_num_rows);
      p.partition_kv = false;
      T *tmp_v = nullptr;
      float *tmp_s = nullptr;
      if (info.split_kv) {
        p.merge_indptr = at<int32_t>(ws.int_buffer, info.merge_indptr_offset);
        tmp_v = at<T>(ws.float_buffer, info.v_offset);
        tmp_s = at<float>(ws.float_buffer, info.s_offset);
      }
      cudaError_t e = cudaSuccess;
      DISPATCH_CTA_TILE_Q(info.cta_tile_q, CTA_TILE_Q, {
        e = flashinfer::BatchPrefillWithPagedKVCacheDispatched<CTA_TILE_Q, D, D, PosEncodingMode::kNone,
                                                               /*use_fp16_qk_reduction=*/false, MaskMode::kCausal,
                                                               Variant, Params>(p, tmp_v, tmp_s,
                                                                                /*enable_pdl=*/false, stream);
      });
      if (e != cudaSuccess) return cuda_error("attention prefill", e);
      return std::string();
    });
  });
}

}  // namespace fi
}  // namespace yllang
