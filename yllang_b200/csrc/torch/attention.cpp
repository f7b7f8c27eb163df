// yllang::Attention and its per-step AttentionContext: the layer glue of the
// reference's Attention (src/include/layers/attention.h:22-68) over the paged
// pool of MHAKVCache, with flashinfer's paged decode / causal prefill kernels
// (attention_fi.cu) as the attention itself.
#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAStream.h>

#include <cmath>
#include <mutex>

#include "attention_fi.h"
#include "yllang_kvpath.h"

namespace yllang {
namespace {

constexpr int64_t kIntWorkspaceBytes = 8ll << 20;  // the plan's request / tile lists

cudaStream_t current_stream(const torch::Device &device) {
  return c10::cuda::getCurrentCUDAStream(device.index()).stream();
}

fi::DType fi_dtype(torch::Dtype t) { return t == torch::kFloat16 ? fi::DType::kFP16 : fi::DType::kBF16; }

std::mutex g_ctx_mu;
std::shared_ptr<AttentionContext> g_ctx;

}  // namespace

struct AttentionContext::Impl {
  torch::Tensor float_ws;  // device
  torch::Tensor int_ws;    // device
  torch::Tensor int_host;  // page-locked host
  std::vector<int64_t> plan;
  int64_t rows{0};         // qo_indptr[B]: query rows of the step

  fi::Workspace workspace() const {
    return fi::Workspace{float_ws.data_ptr(), static_cast<size_t>(float_ws.numel()), int_ws.data_ptr(),
                         int_host.data_ptr(), static_cast<size_t>(int_ws.numel())};
  }
};

// "cuda" names the current device: pin the index so device comparisons hold.
static torch::Device with_index(torch::Device device) {
  if (device.is_cuda() && !device.has_index())
    return torch::Device(torch::kCUDA, static_cast<c10::DeviceIndex>(c10::cuda::current_device()));
  return device;
}

AttentionContext::AttentionContext(torch::Device device, int64_t workspace_bytes)
    : m_device_(with_index(device)), m_impl_(std::make_unique<Impl>()) {
  RuntimeCheck(device.is_cuda(), "AttentionContext: the device must be a CUDA device");
  RuntimeCheck(workspace_bytes > 0, "AttentionContext: workspace_bytes must be > 0");
  const auto dev = torch::TensorOptions().device(m_device_).dtype(torch::kUInt8);
  m_impl_->float_ws = torch::empty({workspace_bytes}, dev);
  m_impl_->int_ws = torch::empty({kIntWorkspaceBytes}, dev);
  m_impl_->int_host = torch::empty({kIntWorkspaceBytes}, torch::TensorOptions().dtype(torch::kUInt8).pinned_memory(true));
}

AttentionContext::~AttentionContext() = default;

void AttentionContext::Plan(const BatchIndex &index, int num_qo_heads, int num_kv_heads, int head_dim,
                            int page_size, torch::Dtype dtype, std::optional<torch::Tensor> positions) {
  RuntimeCheck(num_qo_heads > 0 && num_kv_heads > 0 && num_qo_heads % num_kv_heads == 0,
               "AttentionContext::Plan: num_qo_heads must be a positive multiple of num_kv_heads");
  RuntimeCheck(head_dim == 64 || head_dim == 128 || head_dim == 256,
               "AttentionContext::Plan: head_dim must be 64, 128 or 256");
  RuntimeCheck(page_size > 0, "AttentionContext::Plan: page_size must be > 0");
  RuntimeCheck(dtype == torch::kBFloat16 || dtype == torch::kFloat16,
               "AttentionContext::Plan: dtype must be bfloat16 or float16");
  for (const auto *t : {&index.kv_indptr, &index.kv_indices, &index.kv_last_page_len, &index.qo_indptr}) {
    RuntimeCheck(t->defined() && t->device() == m_device_ && t->scalar_type() == torch::kInt32 && t->dim() == 1 &&
                     t->is_contiguous(),
                 "AttentionContext::Plan: the page arrays must be contiguous int32 tensors on the context's device");
  }
  const int64_t B = index.kv_indptr.size(0) - 1;
  RuntimeCheck(B >= 0 && index.qo_indptr.size(0) == B + 1 && index.kv_last_page_len.size(0) >= B,
               "AttentionContext::Plan: kv_indptr, qo_indptr [B+1] and kv_last_page_len [B] disagree");
  if (positions) {
    RuntimeCheck(positions->device() == m_device_ && positions->dim() == 1,
                 "AttentionContext::Plan: positions must be [N] on the context's device");
  }
  // host copies (these wait for the stream, so a previous plan's copies out
  // of the page-locked buffer are done before it is written again)
  const torch::Tensor qo = index.qo_indptr.cpu();
  const torch::Tensor kv = index.kv_indptr.cpu();
  const int32_t *qo_h = qo.data_ptr<int32_t>();
  bool decode = B > 0;
  for (int64_t i = 0; i < B && decode; ++i) decode = qo_h[i + 1] - qo_h[i] == 1;
  m_index_ = index;
  m_positions_ = std::move(positions);
  m_qo_heads_ = num_qo_heads;
  m_kv_heads_ = num_kv_heads;
  m_head_dim_ = head_dim;
  m_page_size_ = page_size;
  m_dtype_ = dtype;
  m_decode_ = decode;
  m_impl_->rows = B > 0 ? qo_h[B] : 0;
  m_impl_->plan.clear();
  m_planned_ = false;
  if (B > 0) {
    const fi::Shape shape{static_cast<int>(B), num_qo_heads, num_kv_heads, head_dim, page_size, fi_dtype(dtype)};
    const std::string err =
        decode ? fi::PlanDecode(m_impl_->workspace(), shape, kv.data_ptr<int32_t>(), current_stream(m_device_),
                                &m_impl_->plan)
               : fi::PlanPrefill(m_impl_->workspace(), shape, qo_h, kv.data_ptr<int32_t>(), current_stream(m_device_),
                                 &m_impl_->plan);
    RuntimeCheck(err.empty(), "AttentionContext::Plan: " + err);
  }
  m_planned_ = true;
}

void SetAttentionContext(std::shared_ptr<AttentionContext> ctx) {
  std::lock_guard<std::mutex> lock(g_ctx_mu);
  g_ctx = std::move(ctx);
}

std::shared_ptr<AttentionContext> GetAttentionContext() {
  std::lock_guard<std::mutex> lock(g_ctx_mu);
  return g_ctx;
}

Attention::Attention(int layer_id, int num_qo_heads, int num_kv_heads, int head_dim,
                     std::shared_ptr<MHAKVCache> cache, QKNormRope norm_rope)
    : m_layer_id_(layer_id), m_head_dim_(head_dim), m_cache_(std::move(cache)), m_norm_rope_(std::move(norm_rope)) {
  RuntimeCheck(m_cache_ != nullptr, "Attention: a KV cache is required");
  const int tp = GetDistributedInfo().GetSize();
  RuntimeCheck(num_qo_heads % tp == 0 && num_kv_heads % tp == 0,
               "Attention: head counts not divisible by the tensor-parallel size");
  m_qo_heads_ = num_qo_heads / tp;
  m_kv_heads_ = num_kv_heads / tp;
  RuntimeCheck(m_kv_heads_ > 0 && m_qo_heads_ % m_kv_heads_ == 0,
               "Attention: query heads must be a multiple of the KV heads");
  RuntimeCheck(layer_id >= 0 && layer_id < m_cache_->NumLayers(), "Attention: layer_id outside the cache's layers");
  RuntimeCheck(m_cache_->NumLocalKVHeads() == m_kv_heads_ && m_cache_->HeadDim() == head_dim,
               "Attention: the cache's KV heads or head_dim differ from the layer's");
  m_fused_ = m_norm_rope_.q_weight.has_value() || m_norm_rope_.k_weight.has_value() ||
             m_norm_rope_.cos_sin_cache.has_value();
}

torch::Tensor Attention::Forward(const torch::Tensor &qkv_raw) {
  const std::shared_ptr<AttentionContext> ctx = GetAttentionContext();
  RuntimeCheck(ctx != nullptr, "Attention::Forward: no attention context is set (SetAttentionContext)");
  return Forward(qkv_raw, *ctx);
}

torch::Tensor Attention::Forward(const torch::Tensor &qkv_raw, const AttentionContext &ctx) {
  RuntimeCheck(ctx.Planned(), "Attention::Forward: the context has no plan for this step");
  RuntimeCheck(ctx.NumQoHeads() == m_qo_heads_ && ctx.NumKvHeads() == m_kv_heads_ && ctx.HeadDim() == m_head_dim_ &&
                   ctx.PageSize() == m_cache_->PageSize(),
               "Attention::Forward: the context was planned for other heads, head_dim or page size");
  const int64_t D = m_head_dim_, Hq = m_qo_heads_, Hk = m_kv_heads_;
  RuntimeCheck(qkv_raw.dim() == 2 && qkv_raw.size(1) == (Hq + 2 * Hk) * D && qkv_raw.stride(1) == 1,
               "Attention::Forward: qkv_raw must be [N, (Hq + 2 Hk) * head_dim] with contiguous rows");
  RuntimeCheck(qkv_raw.device() == m_cache_->Buffer().device() && qkv_raw.device() == ctx.Device(),
               "Attention::Forward: qkv_raw is on another device");
  RuntimeCheck(qkv_raw.scalar_type() == ctx.Dtype() && qkv_raw.scalar_type() == m_cache_->Buffer().scalar_type(),
               "Attention::Forward: qkv_raw's dtype differs from the cache's and the plan's");
  const int64_t N = qkv_raw.size(0);
  RuntimeCheck(N == ctx.Internal().rows, "Attention::Forward: qkv_raw rows differ from the step's new tokens");
  auto out = torch::empty({N, Hq, D}, qkv_raw.options());
  if (N == 0) return out.view({N, Hq * D});
  const torch::Tensor q = qkv_raw.narrow(1, 0, Hq * D).unflatten(1, {Hq, D});
  const torch::Tensor k = qkv_raw.narrow(1, Hq * D, Hk * D).unflatten(1, {Hk, D});
  const torch::Tensor v = qkv_raw.narrow(1, (Hq + Hk) * D, Hk * D).unflatten(1, {Hk, D});
  const torch::Tensor slots = ctx.Index().slot_mapping.narrow(0, 0, N);

  torch::Tensor q_use = q;
  if (m_fused_) {
    QKNormRope opts = m_norm_rope_;
    if (opts.cos_sin_cache) {
      RuntimeCheck(ctx.Positions().has_value(), "Attention::Forward: rotary embedding needs the step's positions");
      opts.positions = ctx.Positions();
    }
    q_use = m_cache_->StoreKVNormRope(q, k, v, slots, m_layer_id_, opts);
  } else {
    m_cache_->StoreKV(k, v, slots, m_layer_id_);
  }

  const torch::Tensor kc = m_cache_->KCache(m_layer_id_);  // [P, ps, Hk, D]
  const torch::Tensor vc = m_cache_->VCache(m_layer_id_);
  const BatchIndex &ix = ctx.Index();
  const fi::PagedPool pool{kc.data_ptr(),
                           vc.data_ptr(),
                           kc.stride(0),
                           kc.stride(1),
                           kc.stride(2),
                           ix.kv_indptr.data_ptr<int32_t>(),
                           ix.kv_indices.data_ptr<int32_t>(),
                           ix.kv_last_page_len.data_ptr<int32_t>()};
  const fi::Rows rows{q_use.data_ptr(), out.data_ptr(), q_use.stride(0), q_use.stride(1), out.stride(0), out.stride(1)};
  const fi::Shape shape{static_cast<int>(ix.kv_indptr.size(0) - 1), static_cast<int>(Hq), static_cast<int>(Hk),
                        static_cast<int>(D), m_cache_->PageSize(), fi_dtype(ctx.Dtype())};
  const float sm_scale = 1.0f / std::sqrt(static_cast<float>(D));
  const cudaStream_t stream = current_stream(qkv_raw.device());
  const std::string err =
      ctx.IsDecode()
          ? fi::RunDecode(ctx.Internal().workspace(), shape, ctx.Internal().plan, rows, pool, sm_scale, stream)
          : fi::RunPrefill(ctx.Internal().workspace(), shape, ctx.Internal().plan, rows,
                           ix.qo_indptr.data_ptr<int32_t>(), pool, sm_scale, stream);
  RuntimeCheck(err.empty(), "Attention::Forward: " + err);
  return out.view({N, Hq * D});
}

}  // namespace yllang
