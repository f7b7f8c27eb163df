// C++17 libtorch front end: validation, views and the host index driver on
// top of the C ABI of libyl_kvpath.so.  See yllang_kvpath.h.
#include "yllang_kvpath.h"

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <c10/core/DeviceGuard.h>

#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <numeric>
#include <sstream>

#include "yl_kvpath.h"

namespace yllang {

void RuntimeCheck(bool cond, const std::string &msg) {
  if (!cond) throw PanicError(msg);
}

bool DeviceErrorChecksEnabled() {
  static const bool on = [] {
    const char *e = std::getenv("YLLANG_CHECK_DEVICE_ERRORS");
    return e != nullptr && *e != '\0' && std::string(e) != "0";
  }();
  return on;
}

std::string DeviceErrorNames(uint32_t bits) {
  static const std::pair<uint32_t, const char *> kNames[] = {
      {YL_DEVERR_SLOT_RANGE, "SLOT_RANGE"},           {YL_DEVERR_PAGE_RANGE, "PAGE_RANGE"},
      {YL_DEVERR_ROW_OVERFLOW, "ROW_OVERFLOW"},       {YL_DEVERR_INDICES_CAP, "INDICES_CAP"},
      {YL_DEVERR_SLOTS_CAP, "SLOTS_CAP"},             {YL_DEVERR_NEGATIVE_LEN, "NEGATIVE_LEN"},
      {YL_DEVERR_INDPTR_OVERFLOW, "INDPTR_OVERFLOW"}, {YL_DEVERR_TABLE_ROW, "TABLE_ROW"},
      {YL_DEVERR_TOKEN_COUNT, "TOKEN_COUNT"},         {YL_DEVERR_TIMEOUT, "TIMEOUT"},
      {YL_DEVERR_INDEX_RANGE, "INDEX_RANGE"},         {YL_DEVERR_POSITION_RANGE, "POSITION_RANGE"},
      {YL_DEVERR_POOL_EMPTY, "POOL_EMPTY"},           {YL_DEVERR_POOL_OVERFLOW, "POOL_OVERFLOW"},
      {YL_DEVERR_DUPLICATE_ROW, "DUPLICATE_ROW"}};
  std::string out;
  for (const auto &[bit, name] : kNames) {
    if ((bits & bit) == 0) continue;
    if (!out.empty()) out += '|';
    out += name;
    bits &= ~bit;
  }
  if (bits != 0) {
    std::ostringstream os;
    os << (out.empty() ? "" : "|") << "0x" << std::hex << bits;
    out += os.str();
  }
  return out;
}

namespace {

// NVTX range over one front-end call, so a profiler timeline (nsys, or ncu's
// --nvtx range filters) shows which call launched which kernels; costs a
// function-pointer check when no tool is attached.
class Range {
 public:
  explicit Range(const char *name) { nvtxRangePushA(name); }
  ~Range() { nvtxRangePop(); }
  Range(const Range &) = delete;
  Range &operator=(const Range &) = delete;
};

void CheckStatus(int status, const char *what) {
  if (status != YL_OK) {
    std::ostringstream os;
    os << what << ": " << yl_status_string(status) << " (" << status << "): " << yl_last_error();
    throw PanicError(os.str());
  }
}

// Debug mode (see DeviceErrorChecksEnabled): a call given no device error
// word runs with a private one; Check() then waits for the stream and throws
// PanicError naming the bits the kernels raised.
class DeviceErrorScope {
 public:
  DeviceErrorScope(const torch::Device &device, uint32_t *given, const char *what) : m_word_(given), m_what_(what) {
    if (given == nullptr && DeviceErrorChecksEnabled()) {
      m_private_ = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(device));
      m_word_ = reinterpret_cast<uint32_t *>(m_private_.data_ptr<int32_t>());
    }
  }
  uint32_t *word() const { return m_word_; }
  void Check() const {
    if (!m_private_.defined()) return;
    const auto bits = static_cast<uint32_t>(m_private_.item<int32_t>());
    if (bits != 0) {
      std::ostringstream os;
      os << m_what_ << ": device error bits 0x" << std::hex << bits << std::dec << " (" << DeviceErrorNames(bits)
         << ")";
      throw PanicError(os.str());
    }
  }

 private:
  torch::Tensor m_private_;
  uint32_t *m_word_;
  const char *m_what_;
};

// A caller's device error word: a 4-byte tensor on the call's device.
uint32_t *ErrorWordOf(const std::optional<torch::Tensor> &w, const torch::Device &device, const char *what) {
  if (!w) return nullptr;
  RuntimeCheck(w->numel() >= 1 && w->element_size() == 4 && w->device() == device,
               std::string(what) + ": error_word must be a 4-byte tensor on the call's CUDA device");
  return static_cast<uint32_t *>(w->data_ptr());
}

cudaStream_t CurrentStream(const torch::Tensor &t) {
  return reinterpret_cast<cudaStream_t>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void CheckSameDeviceDtype(const torch::Tensor &ref, std::initializer_list<const torch::Tensor *> ts,
                          const char *what) {
  RuntimeCheck(ref.is_cuda(), std::string(what) + ": tensors must be CUDA tensors");
  for (const auto *t : ts) {
    RuntimeCheck(t->device() == ref.device(), std::string(what) + ": tensors on different devices");
    RuntimeCheck(t->scalar_type() == ref.scalar_type(), std::string(what) + ": tensors of different dtypes");
  }
}

// Store with explicit layer count; shapes already checked by the callers.
void LaunchStore(const torch::Tensor &k, const torch::Tensor &v, const torch::Tensor &k_cache,
                 const torch::Tensor &v_cache, const torch::Tensor &indices, int64_t num_layers, int64_t num_slots,
                 uint32_t *error_word) {
  const int64_t n = indices.size(0);
  if (n == 0) return;  // MHAKVCache::StoreKV returns early (mha_kvcache.h:77-79)
  const int64_t item = k.element_size();
  const bool multi = num_layers > 1 || k.dim() == 3;
  yl_store_args a{};
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.slots = indices.data_ptr();
  a.slot_is_int64 = indices.scalar_type() == torch::kInt64 ? 1 : 0;
  a.num_layers = static_cast<int32_t>(num_layers);
  a.num_tokens = n;
  a.row_bytes = k.size(-1) * item;
  a.k_row_stride = k.stride(-2) * item;
  a.v_row_stride = v.stride(-2) * item;
  a.cache_row_stride = k_cache.stride(-2) * item;
  if (multi) {
    a.k_layer_stride = k.stride(0) * item;
    a.v_layer_stride = v.stride(0) * item;
    a.cache_layer_stride = k_cache.stride(0) * item;
  }
  a.num_slots = num_slots;
  const DeviceErrorScope errors(k.device(), error_word, "yl_kv_store");
  a.error_word = errors.word();
  const c10::cuda::CUDAGuard guard(k.device());
  CheckStatus(yl_kv_store(&a, CurrentStream(k)), "yl_kv_store");
  errors.Check();
}

void CheckIndices(const torch::Tensor &indices, int64_t n, const torch::Tensor &k) {
  RuntimeCheck(indices.dim() == 1 && indices.size(0) == n, "StoreKVCache: indices must be [N]");
  RuntimeCheck(n <= 1 || indices.stride(0) == 1, "StoreKVCache: indices must have stride [1]");
  RuntimeCheck(indices.scalar_type() == torch::kInt32 || indices.scalar_type() == torch::kInt64,
               "StoreKVCache: indices must be int32 or int64");
  RuntimeCheck(indices.device() == k.device(), "StoreKVCache: indices on a different device");
}

}  // namespace

void StoreKVCache(const torch::Tensor &k, const torch::Tensor &v, const torch::Tensor &k_cache,
                  const torch::Tensor &v_cache, const torch::Tensor &indices) {
  const Range range("yllang::StoreKVCache");
  // TensorMatcher contract of store_kv_cache.cu:108-124
  RuntimeCheck(k_cache.dim() == 2 && v_cache.dim() == 2, "StoreKVCache: caches must be [S, E]");
  RuntimeCheck(k.dim() == 2 && v.dim() == 2, "StoreKVCache: k and v must be [N, E]");
  RuntimeCheck(k_cache.sizes() == v_cache.sizes() && k_cache.strides() == v_cache.strides(),
               "StoreKVCache: k_cache and v_cache differ in shape or stride");
  RuntimeCheck(k.sizes() == v.sizes(), "StoreKVCache: k and v differ in shape");
  RuntimeCheck(k.size(1) == k_cache.size(1), "StoreKVCache: row size of inputs and caches differ");
  RuntimeCheck(k.stride(1) == 1 && v.stride(1) == 1 && k_cache.stride(1) == 1,
               "StoreKVCache: rows must be contiguous (stride [*, 1])");
  CheckSameDeviceDtype(k, {&v, &k_cache, &v_cache}, "StoreKVCache");
  CheckIndices(indices, k.size(0), k);
  LaunchStore(k, v, k_cache, v_cache, indices, 1, k_cache.size(0), nullptr);
}

void StoreKVCacheLayers(const torch::Tensor &k, const torch::Tensor &v, const torch::Tensor &k_cache,
                        const torch::Tensor &v_cache, const torch::Tensor &indices) {
  const Range range("yllang::StoreKVCacheLayers");
  RuntimeCheck(k.dim() == 3 && v.dim() == 3, "StoreKVCacheLayers: k and v must be [L, N, E]");
  RuntimeCheck(k_cache.dim() == 3 && v_cache.dim() == 3, "StoreKVCacheLayers: caches must be [L, S, E]");
  RuntimeCheck(k.sizes() == v.sizes(), "StoreKVCacheLayers: k and v differ in shape");
  RuntimeCheck(k_cache.sizes() == v_cache.sizes() && k_cache.strides() == v_cache.strides(),
               "StoreKVCacheLayers: k_cache and v_cache differ in shape or stride");
  RuntimeCheck(k.size(0) == k_cache.size(0), "StoreKVCacheLayers: layer counts differ");
  RuntimeCheck(k.size(2) == k_cache.size(2), "StoreKVCacheLayers: row size of inputs and caches differ");
  RuntimeCheck(k.stride(2) == 1 && v.stride(2) == 1 && k_cache.stride(2) == 1,
               "StoreKVCacheLayers: rows must be contiguous");
  CheckSameDeviceDtype(k, {&v, &k_cache, &v_cache}, "StoreKVCacheLayers");
  CheckIndices(indices, k.size(1), k);
  LaunchStore(k, v, k_cache, v_cache, indices, k.size(0), k_cache.size(1), nullptr);
}

void Index(const torch::Tensor &indices, const torch::Tensor &weights, const torch::Tensor &destination) {
  const Range range("yllang::Index");
  RuntimeCheck(weights.dim() == 2 && weights.stride(1) == 1, "Index: weights must be [V, E] with stride [*, 1]");
  RuntimeCheck(destination.dim() == 2 && destination.stride(1) == 1 && destination.size(1) == weights.size(1),
               "Index: destination must be [N, E] with stride [*, 1]");
  CheckSameDeviceDtype(weights, {&destination}, "Index");
  RuntimeCheck(indices.dim() == 1 && indices.size(0) == destination.size(0), "Index: indices must be [N]");
  RuntimeCheck(indices.size(0) <= 1 || indices.stride(0) == 1, "Index: indices must have stride [1]");
  RuntimeCheck(indices.scalar_type() == torch::kInt32 || indices.scalar_type() == torch::kInt64,
               "Index: indices must be int32 or int64");
  RuntimeCheck(indices.device() == weights.device(), "Index: indices on a different device");
  if (indices.size(0) == 0) return;
  const int64_t item = weights.element_size();
  yl_gather_args a{};
  a.table = weights.data_ptr();
  a.out = destination.data_ptr();
  a.indices = indices.data_ptr();
  a.index_is_int64 = indices.scalar_type() == torch::kInt64 ? 1 : 0;
  a.num_indices = indices.size(0);
  a.row_bytes = weights.size(1) * item;
  a.table_row_stride = weights.stride(0) * item;
  a.out_row_stride = destination.stride(0) * item;
  a.num_rows = weights.size(0);
  const DeviceErrorScope errors(weights.device(), nullptr, "yl_gather_rows");
  a.error_word = errors.word();
  const c10::cuda::CUDAGuard guard(weights.device());
  CheckStatus(yl_gather_rows(&a, CurrentStream(weights)), "yl_gather_rows");
  errors.Check();
}

void QKNormRopeStoreKV(const torch::Tensor &q, const torch::Tensor &k, const torch::Tensor &v,
                       const torch::Tensor &k_cache, const torch::Tensor &v_cache, const torch::Tensor &indices,
                       const QKNormRope &opts, const torch::Tensor &q_out) {
  const Range range("yllang::QKNormRopeStoreKV");
  const auto heads_ok = [](const torch::Tensor &t) { return t.dim() == 3 && t.stride(2) == 1 && t.stride(1) == t.size(2); };
  RuntimeCheck(heads_ok(q) && heads_ok(k) && heads_ok(v) && heads_ok(q_out),
               "QKNormRopeStoreKV: q, k, v, q_out must be [N, heads, D] with contiguous heads");
  const int64_t n = q.size(0), hq = q.size(1), d = q.size(2), hk = k.size(1);
  RuntimeCheck(k.sizes() == v.sizes() && k.size(0) == n && k.size(2) == d && q_out.sizes() == q.sizes(),
               "QKNormRopeStoreKV: shapes of q, k, v, q_out disagree");
  RuntimeCheck(q.scalar_type() == torch::kBFloat16 || q.scalar_type() == torch::kHalf,
               "QKNormRopeStoreKV: dtype must be bf16 or fp16");
  CheckSameDeviceDtype(q, {&k, &v, &q_out, &k_cache, &v_cache}, "QKNormRopeStoreKV");
  for (const auto *c : {&k_cache, &v_cache})
    RuntimeCheck(c->dim() == 2 && c->size(1) == hk * d && c->stride(1) == 1,
                 "QKNormRopeStoreKV: caches must be [S, Hk * D] with unit column stride");
  RuntimeCheck(k_cache.sizes() == v_cache.sizes() && k_cache.stride(0) == v_cache.stride(0),
               "QKNormRopeStoreKV: k_cache and v_cache must share shape and row stride");
  RuntimeCheck(indices.dim() == 1 && indices.size(0) == n && (n <= 1 || indices.stride(0) == 1) &&
                   (indices.scalar_type() == torch::kInt32 || indices.scalar_type() == torch::kInt64) &&
                   indices.device() == q.device(),
               "QKNormRopeStoreKV: indices must be contiguous int32/int64 [N] on q's device");
  for (const auto *w : {&opts.q_weight, &opts.k_weight})
    if (*w)
      RuntimeCheck((*w)->dim() == 1 && (*w)->size(0) == d && (*w)->is_contiguous() &&
                       (*w)->scalar_type() == q.scalar_type() && (*w)->device() == q.device(),
                   "QKNormRopeStoreKV: norm weights must be contiguous [D] of q's dtype and device");
  if (opts.cos_sin_cache) {
    const auto &cs = *opts.cos_sin_cache;
    RuntimeCheck(cs.dim() == 2 && cs.size(1) == d && cs.is_contiguous() && cs.scalar_type() == torch::kFloat32 &&
                     cs.device() == q.device(),
                 "QKNormRopeStoreKV: cos_sin_cache must be contiguous fp32 [max_position, D]");
    RuntimeCheck(opts.positions && opts.positions->dim() == 1 && opts.positions->size(0) == n &&
                     (n <= 1 || opts.positions->stride(0) == 1) &&
                     (opts.positions->scalar_type() == torch::kInt32 ||
                      opts.positions->scalar_type() == torch::kInt64) &&
                     opts.positions->device() == q.device(),
                 "QKNormRopeStoreKV: positions must be contiguous int32/int64 [N] on q's device");
  }
  if (n == 0) return;
  const int64_t item = q.element_size();
  yl_qkv_store_args a{};
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.q_out = q_out.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.slots = indices.data_ptr();
  a.q_weight = opts.q_weight ? opts.q_weight->data_ptr() : nullptr;
  a.k_weight = opts.k_weight ? opts.k_weight->data_ptr() : nullptr;
  if (opts.cos_sin_cache) {
    a.cos_sin_cache = opts.cos_sin_cache->data_ptr<float>();
    a.positions = opts.positions->data_ptr();
    a.position_is_int64 = opts.positions->scalar_type() == torch::kInt64 ? 1 : 0;
    a.max_position = opts.cos_sin_cache->size(0);
  }
  a.dtype = q.scalar_type() == torch::kBFloat16 ? YL_DTYPE_BF16 : YL_DTYPE_F16;
  a.slot_is_int64 = indices.scalar_type() == torch::kInt64 ? 1 : 0;
  a.rope_interleaved = opts.interleaved ? 1 : 0;
  a.num_q_heads = static_cast<int32_t>(hq);
  a.num_kv_heads = static_cast<int32_t>(hk);
  a.head_dim = static_cast<int32_t>(d);
  a.eps = static_cast<float>(opts.eps);
  a.num_tokens = n;
  a.q_row_stride = q.stride(0) * item;
  a.k_row_stride = k.stride(0) * item;
  a.v_row_stride = v.stride(0) * item;
  a.q_out_row_stride = q_out.stride(0) * item;
  a.cache_row_stride = k_cache.stride(0) * item;
  a.num_slots = k_cache.size(0);
  const DeviceErrorScope errors(q.device(), nullptr, "yl_qkv_norm_rope_store");
  a.error_word = errors.word();
  const c10::cuda::CUDAGuard guard(q.device());
  CheckStatus(yl_qkv_norm_rope_store(&a, CurrentStream(q)), "yl_qkv_norm_rope_store");
  errors.Check();
}

// ----------------------------------------------------------------------------
DevicePagePool::DevicePagePool(int64_t num_pages, torch::Device device) : m_capacity_(num_pages), m_device_(device) {
  RuntimeCheck(num_pages > 0 && num_pages <= INT32_MAX, "DevicePagePool: num_pages must be in [1, 2^31)");
  RuntimeCheck(device.is_cuda(), "DevicePagePool: the pool lives on a CUDA device");
  if (!m_device_.has_index()) m_device_ = torch::Device(torch::kCUDA, c10::cuda::current_device());
  m_free_pages_ = torch::arange(num_pages, torch::dtype(torch::kInt32).device(device));
  m_free_count_ = torch::full({1}, num_pages, torch::dtype(torch::kInt32).device(device));
}

namespace {
const int32_t *Int32Vector(const torch::Tensor &t, int64_t n, const torch::Device &dev, const char *what) {
  RuntimeCheck(t.dim() == 1 && t.size(0) == n && t.scalar_type() == torch::kInt32 && t.device() == dev &&
                   (n <= 1 || t.stride(0) == 1),
               std::string("DevicePagePool: ") + what + " must be contiguous int32 [n] on the pool's device");
  return t.data_ptr<int32_t>();
}
}  // namespace

void DevicePagePool::Reserve(const torch::Tensor &page_table, const torch::Tensor &prior_len,
                             const torch::Tensor &new_len, int page_size,
                             const std::optional<torch::Tensor> &table_index,
                             const std::optional<torch::Tensor> &error_word) {
  const Range range("yllang::DevicePagePool::Reserve");
  RuntimeCheck(page_table.dim() == 2 && page_table.scalar_type() == torch::kInt32 && page_table.stride(1) == 1 &&
                   page_table.device() == m_device_,
               "DevicePagePool::Reserve: page_table must be int32 [R, W] on the pool's device");
  const int64_t B = prior_len.size(0);
  yl_reserve_args a{};
  a.pool = {m_free_pages_.data_ptr<int32_t>(), m_free_count_.data_ptr<int32_t>(), m_capacity_};
  a.page_table = page_table.data_ptr<int32_t>();
  a.prior_len = Int32Vector(prior_len, B, m_device_, "prior_len");
  a.new_len = Int32Vector(new_len, B, m_device_, "new_len");
  a.table_index = table_index ? Int32Vector(*table_index, B, m_device_, "table_index") : nullptr;
  a.page_table_stride = page_table.stride(0);
  a.num_table_rows = static_cast<int32_t>(page_table.size(0));
  a.max_pages_per_row = static_cast<int32_t>(page_table.size(1));
  a.page_size = page_size;
  a.batch_size = static_cast<int32_t>(B);
  const DeviceErrorScope errors(m_device_, ErrorWordOf(error_word, m_device_, "DevicePagePool::Reserve"),
                                "yl_reserve_pages");
  a.error_word = errors.word();
  const c10::cuda::CUDAGuard guard(m_device_);
  CheckStatus(yl_reserve_pages(&a, c10::cuda::getCurrentCUDAStream(m_device_.index()).stream()), "yl_reserve_pages");
  errors.Check();
}

void DevicePagePool::Release(const torch::Tensor &page_table, const torch::Tensor &rows,
                             const torch::Tensor &num_tokens, int page_size,
                             const std::optional<torch::Tensor> &error_word) {
  const Range range("yllang::DevicePagePool::Release");
  RuntimeCheck(page_table.dim() == 2 && page_table.scalar_type() == torch::kInt32 && page_table.stride(1) == 1 &&
                   page_table.device() == m_device_,
               "DevicePagePool::Release: page_table must be int32 [R, W] on the pool's device");
  const int64_t R = rows.size(0);
  yl_release_args a{};
  a.pool = {m_free_pages_.data_ptr<int32_t>(), m_free_count_.data_ptr<int32_t>(), m_capacity_};
  a.page_table = page_table.data_ptr<int32_t>();
  a.rows = Int32Vector(rows, R, m_device_, "rows");
  a.num_tokens = Int32Vector(num_tokens, R, m_device_, "num_tokens");
  a.page_table_stride = page_table.stride(0);
  a.num_table_rows = static_cast<int32_t>(page_table.size(0));
  a.max_pages_per_row = static_cast<int32_t>(page_table.size(1));
  a.page_size = page_size;
  a.num_release = static_cast<int32_t>(R);
  const DeviceErrorScope errors(m_device_, ErrorWordOf(error_word, m_device_, "DevicePagePool::Release"),
                                "yl_release_pages");
  a.error_word = errors.word();
  const c10::cuda::CUDAGuard guard(m_device_);
  CheckStatus(yl_release_pages(&a, c10::cuda::getCurrentCUDAStream(m_device_.index()).stream()), "yl_release_pages");
  errors.Check();
}

int64_t DevicePagePool::FreeCount() const { return m_free_count_.item<int32_t>(); }

torch::Tensor DevicePagePool::FreeList() const { return m_free_pages_.narrow(0, 0, FreeCount()).clone(); }

DistributedInfo &GetDistributedInfo() {
  static DistributedInfo instance(0, 1);
  return instance;
}

void SetDistributedInfo(int rank, int size) {
  RuntimeCheck(size >= 1 && rank >= 0 && rank < size, "SetDistributedInfo: bad rank/size");
  GetDistributedInfo().SetRank(rank);
  GetDistributedInfo().SetSize(size);
}

// ----------------------------------------------------------------------------
MHAKVCache::MHAKVCache(int num_layers, int num_pages, int num_kv_heads, int head_dim, KVCacheLayout kv_layout,
                       torch::Device device, torch::Dtype dtype, int page_size, bool zero_fill)
    : m_num_layers_(num_layers),
      m_num_pages_(num_pages),
      m_head_dim_(head_dim),
      m_page_size_(page_size),
      m_device_(device) {
  RuntimeCheck(num_layers > 0 && num_pages > 0 && head_dim > 0 && page_size > 0, "MHAKVCache: bad sizes");
  RuntimeCheck(kv_layout == kPageFirst || kv_layout == kLayerFirst, "no such KVCacheLayout");
  const int tp = GetDistributedInfo().GetSize();
  RuntimeCheck(num_kv_heads % tp == 0, "MHAKVCache: num_kv_heads not divisible by the tensor-parallel size");
  m_num_local_kv_heads_ = num_kv_heads / tp;
  const auto options = torch::TensorOptions().device(device).dtype(dtype);
  const std::vector<int64_t> shape{2, num_layers, num_pages, page_size, m_num_local_kv_heads_, head_dim};
  m_buffer_ = zero_fill ? torch::zeros(shape, options) : torch::empty(shape, options);
  const int64_t slots = static_cast<int64_t>(num_pages) * page_size;
  m_k_rows_ = m_buffer_[0].view({num_layers, slots, static_cast<int64_t>(m_num_local_kv_heads_) * head_dim});
  m_v_rows_ = m_buffer_[1].view({num_layers, slots, static_cast<int64_t>(m_num_local_kv_heads_) * head_dim});
}

void MHAKVCache::StoreKV(torch::Tensor k, torch::Tensor v, torch::Tensor loc, int layer_id) {
  RuntimeCheck(layer_id >= 0 && layer_id < m_num_layers_, "MHAKVCache::StoreKV: layer_id out of range");
  RuntimeCheck(loc.dim() == 1, "MHAKVCache::StoreKV: loc must be [N]");
  const int64_t n = loc.size(0);
  if (n == 0) return;
  StoreKVCache(k.view({n, -1}), v.view({n, -1}), m_k_rows_[layer_id], m_v_rows_[layer_id], loc);
}

void MHAKVCache::StoreKVAllLayers(torch::Tensor k, torch::Tensor v, torch::Tensor loc) {
  RuntimeCheck(loc.dim() == 1, "MHAKVCache::StoreKVAllLayers: loc must be [N]");
  const int64_t n = loc.size(0);
  if (n == 0) return;
  RuntimeCheck(k.size(0) == m_num_layers_, "MHAKVCache::StoreKVAllLayers: k must hold every layer");
  StoreKVCacheLayers(k.view({m_num_layers_, n, -1}), v.view({m_num_layers_, n, -1}), m_k_rows_, m_v_rows_, loc);
}

torch::Tensor MHAKVCache::StoreKVNormRope(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor loc,
                                          int layer_id, const QKNormRope &opts, std::optional<torch::Tensor> q_out) {
  RuntimeCheck(layer_id >= 0 && layer_id < m_num_layers_, "MHAKVCache::StoreKVNormRope: layer_id out of range");
  RuntimeCheck(loc.dim() == 1, "MHAKVCache::StoreKVNormRope: loc must be [N]");
  const int64_t n = loc.size(0);
  const auto heads = [&](const torch::Tensor &t) { return t.dim() == 3 ? t : t.view({n, -1, m_head_dim_}); };
  torch::Tensor qh = heads(q), kh = heads(k), vh = heads(v);
  torch::Tensor out = q_out ? heads(*q_out) : torch::empty_like(qh, qh.options().memory_format(at::MemoryFormat::Contiguous));
  QKNormRopeStoreKV(qh, kh, vh, m_k_rows_[layer_id], m_v_rows_[layer_id], loc, opts, out);
  return out;
}

torch::Tensor MHAKVCache::KCache(int layer_id) { return m_buffer_[0][layer_id]; }
torch::Tensor MHAKVCache::VCache(int layer_id) { return m_buffer_[1][layer_id]; }

// ----------------------------------------------------------------------------
BatchIndex BuildBatchIndex(const torch::Tensor &prior_len, const torch::Tensor &new_len,
                           const torch::Tensor &page_table, int page_size,
                           const std::optional<torch::Tensor> &table_index, int64_t num_pages,
                           int64_t kv_indices_capacity, int64_t slot_capacity, torch::Dtype slot_dtype,
                           const std::optional<torch::Tensor> &error_word) {
  const Range range("yllang::BuildBatchIndex");
  RuntimeCheck(prior_len.is_cuda(), "BuildBatchIndex: lengths must be CUDA tensors");
  for (const auto *t : {&prior_len, &new_len, &page_table}) {
    RuntimeCheck(t->scalar_type() == torch::kInt32, "BuildBatchIndex: lengths and page table must be int32");
    RuntimeCheck(t->device() == prior_len.device(), "BuildBatchIndex: tensors on different devices");
  }
  const int64_t B = prior_len.size(0);
  RuntimeCheck(prior_len.dim() == 1 && new_len.dim() == 1 && new_len.size(0) == B,
               "BuildBatchIndex: prior_len and new_len must both be [B]");
  RuntimeCheck(prior_len.is_contiguous() && new_len.is_contiguous(), "BuildBatchIndex: lengths must be contiguous");
  RuntimeCheck(page_table.dim() == 2 && page_table.stride(1) == 1,
               "BuildBatchIndex: page_table must be [R, W] with unit column stride");
  if (table_index) {
    RuntimeCheck(table_index->scalar_type() == torch::kInt32 && table_index->dim() == 1 &&
                     table_index->size(0) == B && table_index->is_contiguous() &&
                     table_index->device() == prior_len.device(),
                 "BuildBatchIndex: table_index must be contiguous int32 [B] on the same device");
  } else {
    RuntimeCheck(page_table.size(0) >= B, "BuildBatchIndex: page_table has fewer rows than the batch");
  }
  RuntimeCheck(slot_dtype == torch::kInt64 || slot_dtype == torch::kInt32, "BuildBatchIndex: slot dtype");
  const int64_t W = page_table.size(1);
  if (kv_indices_capacity < 0 || slot_capacity < 0) {
    const auto tot = prior_len.clamp_min(0).to(torch::kInt64) + new_len.clamp_min(0).to(torch::kInt64);
    if (kv_indices_capacity < 0)
      kv_indices_capacity = torch::clamp_max((tot + page_size - 1).div(page_size, "floor"), W).sum().item<int64_t>();
    if (slot_capacity < 0) slot_capacity = new_len.clamp_min(0).to(torch::kInt64).sum().item<int64_t>();
  }
  const auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(prior_len.device());
  BatchIndex out{torch::empty({B + 1}, i32), torch::empty({kv_indices_capacity}, i32), torch::empty({B}, i32),
                 torch::empty({B + 1}, i32),
                 torch::empty({slot_capacity}, torch::TensorOptions().dtype(slot_dtype).device(prior_len.device()))};
  yl_index_args a{};
  a.prior_len = prior_len.data_ptr<int32_t>();
  a.new_len = new_len.data_ptr<int32_t>();
  a.page_table = page_table.data_ptr<int32_t>();
  a.table_index = table_index ? table_index->data_ptr<int32_t>() : nullptr;
  a.page_table_stride = page_table.stride(0);
  a.num_table_rows = static_cast<int32_t>(page_table.size(0));
  a.max_pages_per_row = static_cast<int32_t>(W);
  a.page_size = page_size;
  a.batch_size = static_cast<int32_t>(B);
  a.slot_is_int64 = slot_dtype == torch::kInt64 ? 1 : 0;
  a.num_pages = num_pages;
  a.kv_indptr = out.kv_indptr.data_ptr<int32_t>();
  a.kv_indices = kv_indices_capacity ? out.kv_indices.data_ptr<int32_t>() : nullptr;
  a.kv_last_page_len = B ? out.kv_last_page_len.data_ptr<int32_t>() : nullptr;
  a.qo_indptr = out.qo_indptr.data_ptr<int32_t>();
  a.slot_mapping = slot_capacity ? out.slot_mapping.data_ptr() : nullptr;
  a.kv_indices_capacity = kv_indices_capacity;
  a.slot_capacity = slot_capacity;
  const DeviceErrorScope errors(prior_len.device(), ErrorWordOf(error_word, prior_len.device(), "BuildBatchIndex"),
                                "yl_build_index");
  a.error_word = errors.word();
  const c10::cuda::CUDAGuard guard(prior_len.device());
  CheckStatus(yl_build_index(&a, CurrentStream(prior_len)), "yl_build_index");
  errors.Check();
  return out;
}

// ----------------------------------------------------------------------------
torch::Tensor Make2DIndices(const torch::Tensor &table, const std::vector<torch::Tensor> &ranges) {
  const Range range("yllang::Make2DIndices");
  RuntimeCheck(table.dim() == 2, "Make2DIndices: table must be 2-D");
  RuntimeCheck(table.is_cuda(), "Make2DIndices: table must be a CUDA tensor (the indices are made on its device)");
  const int64_t R = static_cast<int64_t>(ranges.size());
  std::vector<torch::Tensor> firsts;
  firsts.reserve(ranges.size());
  for (const auto &r : ranges) {
    RuntimeCheck(r.numel() >= 3, "Make2DIndices: each range needs three entries {row, col_start, col_end}");
    RuntimeCheck(r.device() == ranges.front().device(), "Make2DIndices: ranges on different devices");
    firsts.push_back(r.reshape({-1}).narrow(0, 0, 3).to(torch::kInt64));
  }
  const torch::Tensor host = R ? torch::stack(firsts).to(torch::kCPU).contiguous()
                               : torch::empty({0, 3}, torch::dtype(torch::kInt64));
  const int64_t *h = host.data_ptr<int64_t>();
  int64_t total = 0;
  for (int64_t i = 0; i < R; ++i) {
    const int64_t row = h[3 * i], lo = h[3 * i + 1], hi = h[3 * i + 2];
    RuntimeCheck(row >= 0 && lo >= 0 && hi >= lo,
                 "Make2DIndices: a range needs row >= 0, col_start >= 0 and col_end >= col_start");
    RuntimeCheck(row <= INT64_MAX - hi, "Make2DIndices: row + col_end passes INT64_MAX");
    RuntimeCheck(hi - lo < (int64_t{1} << 40) - total, "Make2DIndices: 2^40 indices or more");
    total += hi - lo;
  }
  const auto opts = torch::TensorOptions().dtype(torch::kInt64).device(table.device());
  torch::Tensor out = torch::empty({total}, opts);
  if (total == 0) return out;
  const c10::cuda::CUDAGuard guard(table.device());
  const torch::Tensor dev_ranges = host.to(table.device());
  yl_ranges_args a{};
  a.ranges = dev_ranges.data_ptr<int64_t>();
  a.indices = out.data_ptr<int64_t>();
  a.num_ranges = R;
  a.indices_capacity = total;
  CheckStatus(yl_make_2d_indices(&a, CurrentStream(table)), "yl_make_2d_indices");
  return out;
}

// ----------------------------------------------------------------------------
KVCacheManager::KVCacheManager(int64_t num_pages, int64_t max_requests, int64_t max_pages_per_request,
                               int page_size, torch::Device device)
    : m_num_pages_(num_pages),
      m_max_requests_(max_requests),
      m_max_pages_(max_pages_per_request),
      m_page_size_(page_size),
      m_device_(device) {
  RuntimeCheck(num_pages > 0 && num_pages <= INT32_MAX && max_requests > 0 && max_pages_per_request > 0 &&
                   page_size > 0,
               "KVCacheManager: bad sizes");
  // the free list is page ids 0..P-1 in order and allocation takes its tail
  // (cache_manager.h:33-34, 121-123), the order the device pool keeps too
  m_free_pages_.resize(static_cast<size_t>(num_pages));
  for (int64_t i = 0; i < num_pages; ++i) m_free_pages_[static_cast<size_t>(i)] = static_cast<int32_t>(i);
  m_free_rows_.resize(static_cast<size_t>(max_requests));
  for (int64_t i = 0; i < max_requests; ++i) m_free_rows_[static_cast<size_t>(i)] = max_requests - 1 - i;
  m_row_pages_.assign(static_cast<size_t>(max_requests), 0);
  m_host_table_ = torch::full({max_requests, max_pages_per_request}, -1, torch::dtype(torch::kInt32));
  m_page_table_ = m_host_table_.to(device);
}

int64_t KVCacheManager::AllocateTableSlot() {
  TORCH_CHECK(!m_free_rows_.empty(), "no enough table slots");
  const int64_t row = m_free_rows_.back();
  m_free_rows_.pop_back();
  return row;
}

torch::Tensor KVCacheManager::AllocatePages(int64_t n) {
  TORCH_CHECK(n >= 0 && static_cast<size_t>(n) <= m_free_pages_.size(), "not enough pages");
  // the last n entries of the list, in order (AllocateIndices, cache_manager.h:121-123)
  auto out = torch::empty({n}, torch::dtype(torch::kInt32));
  auto *p = out.data_ptr<int32_t>();
  const size_t keep = m_free_pages_.size() - static_cast<size_t>(n);
  for (int64_t i = 0; i < n; ++i) p[i] = m_free_pages_[keep + static_cast<size_t>(i)];
  m_free_pages_.resize(keep);
  return out;
}

void KVCacheManager::FreePages(const torch::Tensor &pages) {
  const auto c = pages.to(torch::kCPU, torch::kInt32).contiguous();
  const auto *p = c.data_ptr<int32_t>();
  for (int64_t i = 0; i < c.numel(); ++i) {
    TORCH_CHECK(p[i] >= 0 && p[i] < m_num_pages_, "FreePages: page id out of range");
    m_free_pages_.push_back(p[i]);
  }
}

int64_t KVCacheManager::PagesInRow(int64_t table_index) const {
  TORCH_CHECK(table_index >= 0 && table_index < m_max_requests_, "table index out of range");
  return m_row_pages_[static_cast<size_t>(table_index)];
}

torch::Tensor KVCacheManager::Reserve(int64_t table_index, int64_t tokens) {
  TORCH_CHECK(table_index >= 0 && table_index < m_max_requests_, "table index out of range");
  TORCH_CHECK(tokens >= 0, "negative token count");
  const int64_t need = (tokens + m_page_size_ - 1) / m_page_size_;
  TORCH_CHECK(need <= m_max_pages_, "request needs more pages than a page-table row holds");
  int64_t &have = m_row_pages_[static_cast<size_t>(table_index)];
  if (need <= have) return torch::empty({0}, torch::dtype(torch::kInt32));
  auto fresh = AllocatePages(need - have);
  auto *row = m_host_table_.data_ptr<int32_t>() + table_index * m_max_pages_;
  const auto *p = fresh.data_ptr<int32_t>();
  for (int64_t j = have; j < need; ++j) {
    row[j] = p[j - have];
    m_dirty_.push_back(table_index * m_max_pages_ + j);
  }
  have = need;
  return fresh;
}

void KVCacheManager::Release(int64_t table_index) {
  TORCH_CHECK(table_index >= 0 && table_index < m_max_requests_, "table index out of range");
  int64_t &have = m_row_pages_[static_cast<size_t>(table_index)];
  auto *row = m_host_table_.data_ptr<int32_t>() + table_index * m_max_pages_;
  for (int64_t j = 0; j < have; ++j) {
    m_free_pages_.push_back(row[j]);
    row[j] = -1;
    m_dirty_.push_back(table_index * m_max_pages_ + j);
  }
  have = 0;
  m_free_rows_.push_back(table_index);
}

void KVCacheManager::SyncPageTable() {
  const Range range("yllang::KVCacheManager::SyncPageTable");
  if (m_dirty_.empty()) return;
  std::sort(m_dirty_.begin(), m_dirty_.end());
  m_dirty_.erase(std::unique(m_dirty_.begin(), m_dirty_.end()), m_dirty_.end());
  const int64_t n = static_cast<int64_t>(m_dirty_.size());
  const bool cuda = m_device_.is_cuda();
  auto idx = torch::empty({n}, torch::dtype(torch::kInt64).pinned_memory(cuda));
  auto val = torch::empty({n}, torch::dtype(torch::kInt32).pinned_memory(cuda));
  const auto *host = m_host_table_.data_ptr<int32_t>();
  auto *pi = idx.data_ptr<int64_t>();
  auto *pv = val.data_ptr<int32_t>();
  for (int64_t i = 0; i < n; ++i) {
    pi[i] = m_dirty_[static_cast<size_t>(i)];
    pv[i] = host[pi[i]];
  }
  // one scatter of the changed entries; asynchronous on the current stream
  // (the pinned staging buffers stay reserved until the copies have run)
  const c10::OptionalDeviceGuard guard(cuda ? std::optional<c10::Device>(m_device_) : std::nullopt);
  m_page_table_.view({-1}).index_put_({idx.to(m_device_, /*non_blocking=*/cuda)}, val.to(m_device_, cuda));
  m_dirty_.clear();
}

// ----------------------------------------------------------------------------
Batch BatchManager::NextBatch(const std::vector<RequestSlot> &requests) {
  const Range range("yllang::BatchManager::NextBatch");
  auto &cache = *m_cache_;
  const int64_t B = static_cast<int64_t>(requests.size());
  int64_t pages = 0, tokens = 0;
  auto stage = torch::empty({3, std::max<int64_t>(B, 1)}, torch::dtype(torch::kInt32).pinned_memory(true));
  auto *prior = stage.data_ptr<int32_t>();
  auto *fresh = prior + stage.size(1);
  auto *rows = fresh + stage.size(1);
  for (int64_t i = 0; i < B; ++i) {
    const auto &r = requests[static_cast<size_t>(i)];
    TORCH_CHECK(r.cached_len >= 0 && r.cached_len <= r.device_len, "request with cached_len > device_len");
    TORCH_CHECK(r.device_len <= INT32_MAX, "request longer than 2^31 tokens");
    cache.Reserve(r.table_index, r.device_len);
    prior[i] = static_cast<int32_t>(r.cached_len);
    fresh[i] = static_cast<int32_t>(r.device_len - r.cached_len);
    rows[i] = static_cast<int32_t>(r.table_index);
    pages += (r.device_len + cache.PageSize() - 1) / cache.PageSize();
    tokens += r.device_len - r.cached_len;
  }
  cache.SyncPageTable();
  const auto dev = cache.PageTable().device();
  const c10::cuda::CUDAGuard guard(dev);
  auto d = stage.to(dev, /*non_blocking=*/true);
  Batch out;
  out.table_index = d[2].narrow(0, 0, B);
  out.index = BuildBatchIndex(d[0].narrow(0, 0, B), d[1].narrow(0, 0, B), cache.PageTable(), cache.PageSize(),
                              out.table_index, cache.NumPages(), pages, tokens);
  out.num_tokens = tokens;
  return out;
}

}  // namespace yllang
