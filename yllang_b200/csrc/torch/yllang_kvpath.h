// C++17 libtorch front end of the paged KV store and batch index build.
//
// Same names, argument meanings and error behaviour as the reference's
// interfaces on this path, so YLLang-style callers drop in:
//   StoreKVCache<kElementSize>   src/include/kvcache/store_kv_cache.h:29-31
//   BaseKVCache / MHAKVCache     src/include/kvcache/base_kvcache.h:26-70,
//                                src/include/kvcache/mha_kvcache.h:25-148
//   DistributedInfo              src/include/distributed/info.h:18-66
//   KVCacheManager (pages)       src/include/kvcache/cache_manager.h:21-185
//   BatchManager::NextBatch      src/include/batch/batch_manager.h:83-115
// Every device operation goes through the C ABI of libyl_kvpath.so
// (include/yl_kvpath.h) on the current c10 CUDA stream; contract violations
// throw PanicError before any launch, as RuntimeCheck does in the reference.
#pragma once

#include <torch/torch.h>

#include <cstdint>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

namespace yllang {

class PanicError final : public std::runtime_error {
 public:
  explicit PanicError(const std::string &msg) : std::runtime_error(msg) {}
};

// Throws PanicError(msg) when cond is false.
void RuntimeCheck(bool cond, const std::string &msg);

// Debug mode, off by default: YLLANG_CHECK_DEVICE_ERRORS=1 in the environment
// (read once per process).  Every front-end call that is given no device
// error word then runs its kernels with a private one, waits for the stream
// and throws PanicError naming the bits they raised (a slot or page id out of
// range, a short page-table row, a full pool, ...) — the host-side check of
// what the kernels otherwise skip and only flag.  It makes every call
// synchronous.
bool DeviceErrorChecksEnabled();
// "SLOT_RANGE|PAGE_RANGE" for a device error word (YL_DEVERR_* bits).
std::string DeviceErrorNames(uint32_t bits);

// ----------------------------------------------------------------------------
// Store
// ----------------------------------------------------------------------------

// k_cache[indices[i]] <- k[i], v_cache[indices[i]] <- v[i] for i < N, with the
// row size taken at run time.  Shapes as the reference's TensorMatcher
// enforces (store_kv_cache.cu:108-124): caches [S, E] with stride [cs, 1],
// k/v [N, E] with stride [ks, 1], indices [N] int32 or int64 with stride 1,
// one device, one dtype.  An empty batch is a no-op.
void StoreKVCache(const torch::Tensor &k, const torch::Tensor &v, const torch::Tensor &k_cache,
                  const torch::Tensor &v_cache, const torch::Tensor &indices);

// The reference's compile-time-row-size signature; checks
// kElementSize == E * itemsize (store_kv_cache.cu:136) and forwards.
template <size_t kElementSize, size_t kThreadsPreBlock = 128, bool kUsePDL = false>
void StoreKVCache(const torch::Tensor &k, const torch::Tensor &v, const torch::Tensor &k_cache,
                  const torch::Tensor &v_cache, const torch::Tensor &indices) {
  RuntimeCheck(k.dim() == 2 && static_cast<size_t>(k.size(1) * k.element_size()) == kElementSize,
               "StoreKVCache: kElementSize != row elements * dtype size");
  StoreKVCache(k, v, k_cache, v_cache, indices);
}

// Every layer of one step in one launch: k/v [L, N, E], caches [L, S, E].
void StoreKVCacheLayers(const torch::Tensor &k, const torch::Tensor &v, const torch::Tensor &k_cache,
                        const torch::Tensor &v_cache, const torch::Tensor &indices);

// ----------------------------------------------------------------------------
// Row gather (the embedding lookup): destination[i] <- weights[indices[i]].
// Contract of src/layers/index.cu:104-119: weights [V, E] with stride [ws, 1],
// destination [N, E] with stride [ds, 1], indices [N] int32 or int64, one
// device, one dtype.  Out-of-range indices give zero rows.
// ----------------------------------------------------------------------------
void Index(const torch::Tensor &indices, const torch::Tensor &weights, const torch::Tensor &destination);

template <size_t kElementSize, size_t kThreadsPreBlock = 128, bool kUsePDL = false>
void Index(const torch::Tensor &indices, const torch::Tensor &weights, const torch::Tensor &destination) {
  RuntimeCheck(weights.dim() == 2 && static_cast<size_t>(weights.size(1) * weights.element_size()) == kElementSize,
               "Index: kElementSize != row elements * dtype size");
  Index(indices, weights, destination);
}

// ----------------------------------------------------------------------------
// One layer's attention input, fused (see yl_qkv_norm_rope_store): per-head
// RMSNorm of q and k (weights [D]; none given: no norm), rotary embedding from
// cos_sin_cache [max_position, D] fp32 by positions [N] (none: no rotation),
// q written to q_out, k/v stored into the pool rows k_cache/v_cache [S, Hk*D]
// at indices.  q [N, Hq, D], k/v [N, Hk, D], bf16 or fp16, token rows may be
// strided.  The norm is flashinfer::norm::QKRMSNorm's (src/layers/rsm_norm.cu:49).
// ----------------------------------------------------------------------------
struct QKNormRope {
  std::optional<torch::Tensor> q_weight;
  std::optional<torch::Tensor> k_weight;
  double eps{1e-6};
  std::optional<torch::Tensor> cos_sin_cache;
  std::optional<torch::Tensor> positions;
  bool interleaved{false};
};
void QKNormRopeStoreKV(const torch::Tensor &q, const torch::Tensor &k, const torch::Tensor &v,
                       const torch::Tensor &k_cache, const torch::Tensor &v_cache, const torch::Tensor &indices,
                       const QKNormRope &opts, const torch::Tensor &q_out);

// ----------------------------------------------------------------------------
// Tensor-parallel rank info (only the head split uses it)
// ----------------------------------------------------------------------------
class DistributedInfo {
 public:
  DistributedInfo(int rank, int size) noexcept : m_rank_(rank), m_size_(size) {}
  int GetRank() const { return m_rank_; }
  int GetSize() const { return m_size_; }
  void SetRank(int rank) { m_rank_ = rank; }
  void SetSize(int size) { m_size_ = size; }

 private:
  int m_rank_;
  int m_size_;
};
DistributedInfo &GetDistributedInfo();
void SetDistributedInfo(int rank, int size);

// ----------------------------------------------------------------------------
// KV cache
// ----------------------------------------------------------------------------
enum KVCacheLayout : std::uint8_t { kPageFirst = 0, kLayerFirst };

class BaseKVCache {
 public:
  BaseKVCache() = default;
  virtual ~BaseKVCache() = default;
  virtual void StoreKV(torch::Tensor k, torch::Tensor v, torch::Tensor loc, int layer_id) = 0;
  virtual torch::Tensor KCache(int layer_id) = 0;
  virtual torch::Tensor VCache(int layer_id) = 0;
  virtual int NumLayers() = 0;
  virtual torch::Device Device() = 0;
};

// Paged pool [2, L, P, page_size, H_local, D] (layer-major NHD, the layout
// both of the reference's KVCacheLayout values end up with, mha_kvcache.h:53-58),
// H_local = num_kv_heads / tp size.  A slot is page * page_size + offset; the
// per-layer views are [P, page_size, H_local, D] (what a flashinfer NHD paged
// call takes).  page_size defaults to 1 as in the reference
// (mha_kvcache.h:144).
class MHAKVCache : public BaseKVCache {
 public:
  MHAKVCache(int num_layers, int num_pages, int num_kv_heads, int head_dim, KVCacheLayout kv_layout,
             torch::Device device, torch::Dtype dtype, int page_size = 1, bool zero_fill = true);

  // Per-layer store (the reference's call): k, v [..., H_local, D] with N rows.
  void StoreKV(torch::Tensor k, torch::Tensor v, torch::Tensor loc, int layer_id) override;
  // All layers at once: k, v [L, N, H_local * D] (or [L, N, H_local, D]).
  void StoreKVAllLayers(torch::Tensor k, torch::Tensor v, torch::Tensor loc);
  // Q/K norm + rotary embedding + store of one layer (QKNormRopeStoreKV on
  // this layer's pool rows); returns q_out ([N, Hq, D], a new tensor unless given).
  torch::Tensor StoreKVNormRope(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor loc, int layer_id,
                                const QKNormRope &opts, std::optional<torch::Tensor> q_out = std::nullopt);

  torch::Tensor KCache(int layer_id) override;
  torch::Tensor VCache(int layer_id) override;
  int NumLayers() override { return m_num_layers_; }
  torch::Device Device() override { return m_device_; }

  int PageSize() const { return m_page_size_; }
  int NumPages() const { return m_num_pages_; }
  int NumLocalKVHeads() const { return m_num_local_kv_heads_; }
  int HeadDim() const { return m_head_dim_; }
  int64_t NumSlots() const { return static_cast<int64_t>(m_num_pages_) * m_page_size_; }
  torch::Tensor Buffer() const { return m_buffer_; }

 private:
  torch::Tensor m_buffer_;    // [2, L, P, ps, H_local, D]
  torch::Tensor m_k_rows_;    // [L, P*ps, H_local*D] view of K
  torch::Tensor m_v_rows_;    // [L, P*ps, H_local*D] view of V
  int m_num_layers_;
  int m_num_pages_;
  int m_num_local_kv_heads_{0};
  int m_head_dim_;
  int m_page_size_;
  torch::Device m_device_;
};

// ----------------------------------------------------------------------------
// Index build
// ----------------------------------------------------------------------------
struct BatchIndex {
  torch::Tensor kv_indptr;         // int32 [B+1]
  torch::Tensor kv_indices;        // int32 [sum of pages]
  torch::Tensor kv_last_page_len;  // int32 [B]
  torch::Tensor qo_indptr;         // int32 [B+1]
  torch::Tensor slot_mapping;      // int64 (or int32) [sum of new tokens]
};

// Device tensors in, device tensors out (see yl_build_index).  When the
// capacities are negative they are computed from the lengths, which reads
// the lengths back to the host.
BatchIndex BuildBatchIndex(const torch::Tensor &prior_len, const torch::Tensor &new_len,
                           const torch::Tensor &page_table, int page_size,
                           const std::optional<torch::Tensor> &table_index, int64_t num_pages,
                           int64_t kv_indices_capacity = -1, int64_t slot_capacity = -1,
                           torch::Dtype slot_dtype = torch::kInt64,
                           const std::optional<torch::Tensor> &error_word = std::nullopt);

// Make2DIndices (src/include/batch/batch_manager.h:30-51): for each range
// {row, col_start, col_end} (the first three entries of each tensor, read on
// the host as the reference does), the indices row + c for c in
// [col_start, col_end), concatenated.  Made on the table's device as int64
// (the reference returns a CPU float tensor); the table is otherwise unused,
// as in the reference.  A negative entry or col_end < col_start throws
// PanicError (the reference's size_t arithmetic wraps there).
torch::Tensor Make2DIndices(const torch::Tensor &table, const std::vector<torch::Tensor> &ranges);

// ----------------------------------------------------------------------------
// Page allocator + page table (host free lists, device page table)
// ----------------------------------------------------------------------------
// Plays the role of the reference's KVCacheManager (cache_manager.h:21-185)
// for pages of page_size tokens: free page ids and free table rows are host
// stacks; the page table [max_requests, max_pages_per_request] int32 lives on
// the device, with a host mirror whose changed entries are pushed to the
// device once per batch.  Differences from the reference, which are fixes of
// its defects: page ids 0..num_pages-1 (torch::range is end-inclusive,
// cache_manager.h:33-34), allocated pages leave the free list
// (cache_manager.h:123-124), page ids go into the page table
// (cache_manager.h:153 writes the token pool).
class KVCacheManager {
 public:
  KVCacheManager(int64_t num_pages, int64_t max_requests, int64_t max_pages_per_request, int page_size,
                 torch::Device device);

  int64_t NumPages() const { return m_num_pages_; }
  int PageSize() const { return m_page_size_; }
  int64_t RemainingPageCount() const { return static_cast<int64_t>(m_free_pages_.size()); }
  int64_t RemainingTableSlots() const { return static_cast<int64_t>(m_free_rows_.size()); }

  int64_t AllocateTableSlot();             // throws c10::Error when none is left
  torch::Tensor AllocatePages(int64_t n);  // int32 CPU tensor of n page ids
  void FreePages(const torch::Tensor &pages);

  // Make row `table_index` hold ceil(tokens / page_size) pages, allocating the
  // missing ones; returns the pages newly added.
  torch::Tensor Reserve(int64_t table_index, int64_t tokens);
  // Free every page of the row and the row itself.
  void Release(int64_t table_index);
  int64_t PagesInRow(int64_t table_index) const;

  // Push host-side page-table changes to the device (asynchronous, current stream).
  void SyncPageTable();
  torch::Tensor PageTable() const { return m_page_table_; }  // device [R, W] int32
  torch::Tensor HostPageTable() const { return m_host_table_; }

 private:
  int64_t m_num_pages_;
  int64_t m_max_requests_;
  int64_t m_max_pages_;
  int m_page_size_;
  torch::Device m_device_;
  std::vector<int32_t> m_free_pages_;
  std::vector<int64_t> m_free_rows_;
  std::vector<int64_t> m_row_pages_;      // pages held by each row
  std::vector<int64_t> m_dirty_;          // flat entries of the host table changed since the last sync
  torch::Tensor m_host_table_;            // CPU int32 [R, W]
  torch::Tensor m_page_table_;            // device int32 [R, W]
};

// The same free-page list and page-table updates on the device (see
// yl_reserve_pages / yl_release_pages): the list starts as page ids
// 0..num_pages-1, a request takes the tail of the list in order, released
// pages are appended in row order, so a sequence of Reserve / Release calls
// gives the page table KVCacheManager's Reserve / Release give.  Calls are
// asynchronous on the current stream; FreeCount() reads the count back.
class DevicePagePool {
 public:
  DevicePagePool(int64_t num_pages, torch::Device device);
  void Reserve(const torch::Tensor &page_table, const torch::Tensor &prior_len, const torch::Tensor &new_len,
               int page_size, const std::optional<torch::Tensor> &table_index = std::nullopt,
               const std::optional<torch::Tensor> &error_word = std::nullopt);
  void Release(const torch::Tensor &page_table, const torch::Tensor &rows, const torch::Tensor &num_tokens,
               int page_size, const std::optional<torch::Tensor> &error_word = std::nullopt);
  int64_t FreeCount() const;
  torch::Tensor FreeList() const;  // device int32 [FreeCount()]
  int64_t Capacity() const { return m_capacity_; }

 private:
  int64_t m_capacity_;
  torch::Device m_device_;
  torch::Tensor m_free_pages_;  // device int32 [capacity]
  torch::Tensor m_free_count_;  // device int32 [1]
};

// One request in a batch: the reference Request's table_index, cached_len
// and device_len (src/include/request/request.h:81-92).
struct RequestSlot {
  int64_t table_index;
  int64_t cached_len;
  int64_t device_len;
};

struct Batch {
  BatchIndex index;            // page arrays for attention + slot mapping (out_loc)
  torch::Tensor table_index;   // int32 [B] on the device
  int64_t num_tokens{0};       // sum of device_len - cached_len
};

// Per-step index driver: reserves pages for every request's new tokens,
// pushes the page-table changes, stages the lengths in one host-to-device
// copy and launches the index build.  All device work is asynchronous on the
// current stream.
class BatchManager {
 public:
  explicit BatchManager(std::shared_ptr<KVCacheManager> cache) : m_cache_(std::move(cache)) {}
  Batch NextBatch(const std::vector<RequestSlot> &requests);
  std::shared_ptr<KVCacheManager> Cache() const { return m_cache_; }

 private:
  std::shared_ptr<KVCacheManager> m_cache_;
  torch::Tensor m_host_stage_;    // pinned int32 [3, capacity]
  torch::Tensor m_device_stage_;  // device int32 [3, capacity]
};

// ----------------------------------------------------------------------------
// Attention layer: the reference's Attention (src/include/layers/attention.h:22-68),
// whose Forward is a placeholder returning an empty tensor (:55), made real
// for the paged pool.  Forward(qkv) splits one layer's projected rows
// [N, (Hq + 2 Hk) * D] into q, k and v, stores k and v into the layer's pool
// rows at the step's slots (with the per-head Q/K RMSNorm and rotary
// embedding fused in when the layer has them), and runs flashinfer's paged
// attention (third-party, unchanged) over the pool with the step's page
// arrays: batch decode when every sequence adds one token, causal batch
// prefill otherwise (query t of a sequence with L tokens after the step sits
// at position L - n_new + t).  Hq and Hk are this GPU's heads: the model's
// divided by the tensor-parallel size, as MHAKVCache divides its KV heads.
// ----------------------------------------------------------------------------

// One step's attention plan, shared by every layer of the step.
class AttentionContext {
 public:
  explicit AttentionContext(torch::Device device, int64_t workspace_bytes = 256ll << 20);
  ~AttentionContext();
  AttentionContext(const AttentionContext &) = delete;
  AttentionContext &operator=(const AttentionContext &) = delete;

  // Once per step, after the index build.  Reads qo_indptr and kv_indptr
  // back to the host (flashinfer plans its split of long sequences on the
  // host), so it waits for the current stream.  positions [N] int32/int64
  // are the new tokens' positions for the rotary embedding (needed only when
  // a layer rotates q and k).
  void Plan(const BatchIndex &index, int num_qo_heads, int num_kv_heads, int head_dim, int page_size,
            torch::Dtype dtype, std::optional<torch::Tensor> positions = std::nullopt);

  bool Planned() const { return m_planned_; }
  bool IsDecode() const { return m_decode_; }
  const BatchIndex &Index() const { return m_index_; }
  const std::optional<torch::Tensor> &Positions() const { return m_positions_; }
  int NumQoHeads() const { return m_qo_heads_; }
  int NumKvHeads() const { return m_kv_heads_; }
  int HeadDim() const { return m_head_dim_; }
  int PageSize() const { return m_page_size_; }
  torch::Dtype Dtype() const { return m_dtype_; }
  torch::Device Device() const { return m_device_; }

  // flashinfer's workspace and plan (for Attention::Forward).
  struct Impl;
  const Impl &Internal() const { return *m_impl_; }

 private:
  torch::Device m_device_;
  std::unique_ptr<Impl> m_impl_;
  BatchIndex m_index_;
  std::optional<torch::Tensor> m_positions_;
  bool m_planned_{false};
  bool m_decode_{false};
  int m_qo_heads_{0};
  int m_kv_heads_{0};
  int m_head_dim_{0};
  int m_page_size_{0};
  torch::Dtype m_dtype_{torch::kBFloat16};
};

// The context Forward(qkv) uses (the step's, set once per step by its driver).
void SetAttentionContext(std::shared_ptr<AttentionContext> ctx);
std::shared_ptr<AttentionContext> GetAttentionContext();

class Attention {
 public:
  // norm_rope: per-head RMSNorm weights of q and k and/or a cos/sin cache for
  // the rotary embedding (its positions come from the context); empty: the
  // rows are stored and attended as given.
  Attention(int layer_id, int num_qo_heads, int num_kv_heads, int head_dim, std::shared_ptr<MHAKVCache> cache,
            QKNormRope norm_rope = {});

  // qkv_raw [N, (Hq + 2 Hk) * D] (token rows may be strided); returns the
  // attention output [N, Hq * D].
  torch::Tensor Forward(const torch::Tensor &qkv_raw);
  torch::Tensor Forward(const torch::Tensor &qkv_raw, const AttentionContext &ctx);

  int LayerId() const { return m_layer_id_; }
  int NumQoHeads() const { return m_qo_heads_; }
  int NumKvHeads() const { return m_kv_heads_; }

 private:
  int m_layer_id_;
  int m_qo_heads_;  // on this GPU
  int m_kv_heads_;  // on this GPU
  int m_head_dim_;
  std::shared_ptr<MHAKVCache> m_cache_;
  QKNormRope m_norm_rope_;
  bool m_fused_;  // norm and/or rotary applied while storing
};

}  // namespace yllang
