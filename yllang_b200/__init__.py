"""yllang_b200 — B200-native paged KV-cache store and batch index build.

The hot path of one YLLang serving step, rebuilt for sm_100a:

* ``store_kv_cache`` / the C ABI ``yl_kv_store``: scatter the step's new K/V
  rows into the layer-major paged pool by slot mapping (YLLang's
  StoreKVCache / MHAKVCache::StoreKV);
* ``build_index`` / ``yl_build_index``: the batch's kv_indptr, kv_indices,
  kv_last_page_len, qo_indptr and slot_mapping (the index work of YLLang's
  BatchManager::NextBatch), in the paged-KV format flashinfer consumes;
* ``kv_step`` / ``yl_kv_step``: both for one serving step;
* ``gather_rows`` / ``yl_gather_rows``: the embedding-row gather (YLLang's
  Index) on the same copy engine;
* ``qkv_norm_rope_store`` / ``yl_qkv_norm_rope_store``: one layer's Q/K
  RMSNorm and rotary embedding fused with the K/V store;
* ``make_2d_indices`` / ``yl_make_2d_indices``: the flat page-table indices
  of {row, col_start, col_end} ranges (YLLang's Make2DIndices);
* ``DevicePagePool`` / ``yl_reserve_pages``, ``yl_release_pages``: the
  free-page list and page-table updates of YLLang's KVCacheManager on the
  device, feeding the index build without a host round trip.

The kernels live in libyl_kvpath.so (built in-tree); the C++ libtorch front
end with YLLang's class names (MHAKVCache, KVCacheManager, BatchManager,
StoreKVCache) is the extension ``yllang_b200._C`` (``load_extension()``).
"""
from __future__ import annotations

from ._abi import (DEVERR_INDICES_CAP, DEVERR_INDPTR_OVERFLOW, DEVERR_NEGATIVE_LEN, DEVERR_PAGE_RANGE,
                   DEVERR_INDEX_RANGE, DEVERR_ROW_OVERFLOW, DEVERR_SLOT_RANGE, DEVERR_SLOTS_CAP, DEVERR_TABLE_ROW,
                   DEVERR_POOL_EMPTY, DEVERR_POOL_OVERFLOW, DEVERR_POSITION_RANGE, DEVERR_TIMEOUT, DEVERR_TOKEN_COUNT,
                   DEVERR_DUPLICATE_ROW, KVPathError, lib)
from .ops import (BatchIndex, DevicePagePool, PanicError, build_index, gather_rows, kv_step, make_2d_indices,
                  qkv_norm_rope_store, rope_cos_sin_cache, store_args, store_kv_cache)

__all__ = [
    "BatchIndex", "DevicePagePool", "KVPathError", "PanicError", "build_index", "gather_rows", "kv_step", "make_2d_indices",
    "qkv_norm_rope_store",
    "rope_cos_sin_cache", "store_args", "store_kv_cache", "lib",
    "load_extension", "DEVERR_SLOT_RANGE", "DEVERR_PAGE_RANGE", "DEVERR_ROW_OVERFLOW", "DEVERR_INDICES_CAP",
    "DEVERR_SLOTS_CAP", "DEVERR_NEGATIVE_LEN", "DEVERR_INDPTR_OVERFLOW", "DEVERR_TABLE_ROW", "DEVERR_TOKEN_COUNT",
    "DEVERR_TIMEOUT", "DEVERR_INDEX_RANGE", "DEVERR_POSITION_RANGE", "DEVERR_POOL_EMPTY", "DEVERR_POOL_OVERFLOW",
    "DEVERR_DUPLICATE_ROW",
]

_ext = None


def load_extension():
    """Import the C++ libtorch front end yllang_b200._C (built in-tree by
    __graft_entry__.build(); a missing build is an ImportError)."""
    global _ext
    if _ext is None:
        import torch  # noqa: F401  (libtorch must be loaded first)

        from . import _C
        _ext = _C
    return _ext
