// Python bindings of the C++ front end (module yllang_b200._C).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "yllang_kvpath.h"

namespace py = pybind11;
using namespace yllang;

PYBIND11_MODULE(_C, m) {
  m.doc() = "C++17 libtorch front end of the B200 paged KV store and batch index build";
  py::register_exception<PanicError>(m, "PanicError", PyExc_RuntimeError);
  m.def("DeviceErrorChecksEnabled", &DeviceErrorChecksEnabled,
        "true when YLLANG_CHECK_DEVICE_ERRORS was set: calls read their device error bits back and throw");
  m.def("DeviceErrorNames", &DeviceErrorNames, py::arg("bits"), "names of the YL_DEVERR_* bits in a device error word");

  m.def(
      "StoreKVCache",
      [](const torch::Tensor &k, const torch::Tensor &v, const torch::Tensor &kc, const torch::Tensor &vc,
         const torch::Tensor &idx) { StoreKVCache(k, v, kc, vc, idx); },
        py::arg("k"), py::arg("v"), py::arg("k_cache"), py::arg("v_cache"), py::arg("indices"),
        "k_cache[indices[i]] = k[i], v_cache[indices[i]] = v[i] (row size taken at run time)");
  m.def(
      "StoreKVCache2048",
      [](const torch::Tensor &k, const torch::Tensor &v, const torch::Tensor &kc, const torch::Tensor &vc,
         const torch::Tensor &idx) { StoreKVCache<2048>(k, v, kc, vc, idx); },
      py::arg("k"), py::arg("v"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("indices"),
        "the reference's StoreKVCache<kElementSize = 2048> signature (row size checked)");
  m.def("StoreKVCacheLayers", &StoreKVCacheLayers, py::arg("k"), py::arg("v"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("indices"), "every layer of a step in one launch: k, v [L, N, E]");

  m.def(
      "Index",
      [](const torch::Tensor &indices, const torch::Tensor &weights, const torch::Tensor &destination) {
        Index(indices, weights, destination);
      },
      py::arg("indices"), py::arg("weights"), py::arg("destination"),
      "destination[i] = weights[indices[i]] (the embedding lookup of yllang::Index)");

  py::class_<DevicePagePool, std::shared_ptr<DevicePagePool>>(m, "DevicePagePool")
      .def(py::init([](int64_t num_pages, const std::string &device) {
             return std::make_shared<DevicePagePool>(num_pages, torch::Device(device));
           }),
           py::arg("num_pages"), py::arg("device") = "cuda")
      .def("Reserve", &DevicePagePool::Reserve, py::arg("page_table"), py::arg("prior_len"), py::arg("new_len"),
           py::arg("page_size"), py::arg("table_index") = py::none(), py::arg("error_word") = py::none())
      .def("Release", &DevicePagePool::Release, py::arg("page_table"), py::arg("rows"), py::arg("num_tokens"),
           py::arg("page_size"), py::arg("error_word") = py::none())
      .def("FreeCount", &DevicePagePool::FreeCount)
      .def("FreeList", &DevicePagePool::FreeList)
      .def("Capacity", &DevicePagePool::Capacity);

  py::class_<QKNormRope>(m, "QKNormRope")
      .def(py::init<>())
      .def_readwrite("q_weight", &QKNormRope::q_weight)
      .def_readwrite("k_weight", &QKNormRope::k_weight)
      .def_readwrite("eps", &QKNormRope::eps)
      .def_readwrite("cos_sin_cache", &QKNormRope::cos_sin_cache)
      .def_readwrite("positions", &QKNormRope::positions)
      .def_readwrite("interleaved", &QKNormRope::interleaved);
  m.def("QKNormRopeStoreKV", &QKNormRopeStoreKV, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("indices"), py::arg("opts"), py::arg("q_out"));

  m.def("SetDistributedInfo", &SetDistributedInfo, py::arg("rank"), py::arg("size"));
  m.def("GetDistributedInfo", []() {
    const auto &d = GetDistributedInfo();
    return py::make_tuple(d.GetRank(), d.GetSize());
  });

  py::enum_<KVCacheLayout>(m, "KVCacheLayout")
      .value("kPageFirst", kPageFirst)
      .value("kLayerFirst", kLayerFirst)
      .export_values();

  py::class_<MHAKVCache, std::shared_ptr<MHAKVCache>>(m, "MHAKVCache")
      .def(py::init([](int num_layers, int num_pages, int num_kv_heads, int head_dim, KVCacheLayout layout,
                       const std::string &device, py::object dtype, int page_size, bool zero_fill) {
             const auto st = torch::python::detail::py_object_to_dtype(dtype);
             return std::make_shared<MHAKVCache>(num_layers, num_pages, num_kv_heads, head_dim, layout,
                                                 torch::Device(device), st, page_size, zero_fill);
           }),
           py::arg("num_layers"), py::arg("num_pages"), py::arg("num_kv_heads"), py::arg("head_dim"),
           py::arg("kv_layout"), py::arg("device"), py::arg("dtype"), py::arg("page_size") = 1,
           py::arg("zero_fill") = true)
      .def("StoreKV", &MHAKVCache::StoreKV, py::arg("k"), py::arg("v"), py::arg("loc"), py::arg("layer_id"))
      .def("StoreKVAllLayers", &MHAKVCache::StoreKVAllLayers, py::arg("k"), py::arg("v"), py::arg("loc"))
      .def("StoreKVNormRope", &MHAKVCache::StoreKVNormRope, py::arg("q"), py::arg("k"), py::arg("v"),
           py::arg("loc"), py::arg("layer_id"), py::arg("opts"), py::arg("q_out") = py::none())
      .def("KCache", &MHAKVCache::KCache)
      .def("VCache", &MHAKVCache::VCache)
      .def("NumLayers", &MHAKVCache::NumLayers)
      .def("Device", [](MHAKVCache &c) { return c.Device().str(); })
      .def("PageSize", &MHAKVCache::PageSize)
      .def("NumPages", &MHAKVCache::NumPages)
      .def("NumLocalKVHeads", &MHAKVCache::NumLocalKVHeads)
      .def("HeadDim", &MHAKVCache::HeadDim)
      .def("NumSlots", &MHAKVCache::NumSlots)
      .def("Buffer", &MHAKVCache::Buffer);

  py::class_<BatchIndex>(m, "BatchIndex")
      .def_readonly("kv_indptr", &BatchIndex::kv_indptr)
      .def_readonly("kv_indices", &BatchIndex::kv_indices)
      .def_readonly("kv_last_page_len", &BatchIndex::kv_last_page_len)
      .def_readonly("qo_indptr", &BatchIndex::qo_indptr)
      .def_readonly("slot_mapping", &BatchIndex::slot_mapping);

  m.def(
      "BuildBatchIndex",
      [](const torch::Tensor &prior_len, const torch::Tensor &new_len, const torch::Tensor &page_table, int page_size,
         std::optional<torch::Tensor> table_index, int64_t num_pages, int64_t kv_indices_capacity,
         int64_t slot_capacity, bool slot_int64, std::optional<torch::Tensor> error_word) {
        return BuildBatchIndex(prior_len, new_len, page_table, page_size, table_index, num_pages,
                               kv_indices_capacity, slot_capacity, slot_int64 ? torch::kInt64 : torch::kInt32,
                               error_word);
      },
      py::arg("prior_len"), py::arg("new_len"), py::arg("page_table"), py::arg("page_size"),
      py::arg("table_index") = py::none(), py::arg("num_pages") = 0, py::arg("kv_indices_capacity") = -1,
      py::arg("slot_capacity") = -1, py::arg("slot_int64") = true, py::arg("error_word") = py::none());
  m.def("Make2DIndices", &Make2DIndices, py::arg("table"), py::arg("ranges"),
        "flat indices row + c, c in [col_start, col_end), of {row, col_start, col_end} ranges (int64, on the "
        "table's device)");

  py::class_<AttentionContext, std::shared_ptr<AttentionContext>>(m, "AttentionContext")
      .def(py::init([](const std::string &device, int64_t workspace_bytes) {
             return std::make_shared<AttentionContext>(torch::Device(device), workspace_bytes);
           }),
           py::arg("device"), py::arg("workspace_bytes") = 256ll << 20)
      .def(
          "Plan",
          [](AttentionContext &c, const BatchIndex &index, int num_qo_heads, int num_kv_heads, int head_dim,
             int page_size, py::object dtype, std::optional<torch::Tensor> positions) {
            c.Plan(index, num_qo_heads, num_kv_heads, head_dim, page_size,
                   torch::python::detail::py_object_to_dtype(dtype), positions);
          },
          py::arg("index"), py::arg("num_qo_heads"), py::arg("num_kv_heads"), py::arg("head_dim"),
          py::arg("page_size"), py::arg("dtype"), py::arg("positions") = py::none(),
          "plan the step's paged attention from its page arrays (waits for the current stream)")
      .def("IsDecode", &AttentionContext::IsDecode)
      .def("Planned", &AttentionContext::Planned);
  m.def("SetAttentionContext", &SetAttentionContext, py::arg("ctx"));
  m.def("GetAttentionContext", &GetAttentionContext);
  py::class_<Attention, std::shared_ptr<Attention>>(m, "Attention")
      .def(py::init<int, int, int, int, std::shared_ptr<MHAKVCache>, QKNormRope>(), py::arg("layer_id"),
           py::arg("num_qo_heads"), py::arg("num_kv_heads"), py::arg("head_dim"), py::arg("cache"),
           py::arg("norm_rope") = QKNormRope{})
      .def("Forward", py::overload_cast<const torch::Tensor &>(&Attention::Forward), py::arg("qkv_raw"),
           "store this layer's K/V and attend over the pool, with the context set by SetAttentionContext")
      .def("Forward", py::overload_cast<const torch::Tensor &, const AttentionContext &>(&Attention::Forward),
           py::arg("qkv_raw"), py::arg("ctx"))
      .def("LayerId", &Attention::LayerId)
      .def("NumQoHeads", &Attention::NumQoHeads)
      .def("NumKvHeads", &Attention::NumKvHeads);

  py::class_<KVCacheManager, std::shared_ptr<KVCacheManager>>(m, "KVCacheManager")
      .def(py::init([](int64_t num_pages, int64_t max_requests, int64_t max_pages_per_request, int page_size,
                       const std::string &device) {
             return std::make_shared<KVCacheManager>(num_pages, max_requests, max_pages_per_request, page_size,
                                                     torch::Device(device));
           }),
           py::arg("num_pages"), py::arg("max_requests"), py::arg("max_pages_per_request"), py::arg("page_size"),
           py::arg("device"))
      .def("NumPages", &KVCacheManager::NumPages)
      .def("PageSize", &KVCacheManager::PageSize)
      .def("RemainingPageCount", &KVCacheManager::RemainingPageCount)
      .def("RemainingTableSlots", &KVCacheManager::RemainingTableSlots)
      .def("AllocateTableSlot", &KVCacheManager::AllocateTableSlot)
      .def("AllocatePages", &KVCacheManager::AllocatePages)
      .def("FreePages", &KVCacheManager::FreePages)
      .def("Reserve", &KVCacheManager::Reserve)
      .def("Release", &KVCacheManager::Release)
      .def("PagesInRow", &KVCacheManager::PagesInRow)
      .def("SyncPageTable", &KVCacheManager::SyncPageTable)
      .def("PageTable", &KVCacheManager::PageTable)
      .def("HostPageTable", &KVCacheManager::HostPageTable);

  py::class_<RequestSlot>(m, "RequestSlot")
      .def(py::init<int64_t, int64_t, int64_t>(), py::arg("table_index"), py::arg("cached_len"),
           py::arg("device_len"))
      .def_readwrite("table_index", &RequestSlot::table_index)
      .def_readwrite("cached_len", &RequestSlot::cached_len)
      .def_readwrite("device_len", &RequestSlot::device_len);

  py::class_<Batch>(m, "Batch")
      .def_readonly("index", &Batch::index)
      .def_readonly("table_index", &Batch::table_index)
      .def_readonly("num_tokens", &Batch::num_tokens)
      .def_property_readonly("out_loc", [](const Batch &b) { return b.index.slot_mapping; });

  py::class_<BatchManager>(m, "BatchManager")
      .def(py::init<std::shared_ptr<KVCacheManager>>(), py::arg("cache"))
      .def("NextBatch", &BatchManager::NextBatch, py::arg("requests"))
      .def("Cache", &BatchManager::Cache);
}
