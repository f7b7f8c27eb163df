"""Attention glue: the KV path of one attention layer, end to end.

YLLang's `Attention::Forward` is a placeholder (src/include/layers/attention.h:55);
its intended step is: store the layer's new K/V rows into the paged pool, then
run paged attention over the batch's page arrays.  Here that is

* once per step: `yl_build_index` gives kv_indptr / kv_indices /
  kv_last_page_len / slot_mapping, and `plan()` hands the first three to
  flashinfer's paged decode (third-party, unchanged);
* per layer: `forward()` stores the new rows by slot_mapping (`yl_kv_store`)
  and runs flashinfer over the layer's [pages, page_size, kv_heads, head_dim]
  pool views (NHD), which is exactly the pool layout of MHAKVCache.

`PagedDecodeAttention` takes one new token per sequence;
`PagedPrefillAttention` takes any number (prefill, chunked prefill, mixed
batches), with qo_indptr from the same index build and a causal mask aligned
to each sequence's end.

flashinfer compiles its kernels on first use; `prebuild()` (run by the
repository build) compiles the decode kernels into the package's build
folder, which `FLASHINFER_WORKSPACE_BASE` points flashinfer at, so a GPU run
loads them instead of compiling.
"""
from __future__ import annotations

import os

import torch

from .ops import BatchIndex, store_kv_cache

_FI_BASE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build", "fi")
PREFILL_BACKEND = "fa2"  # flashinfer's portable prefill kernels (its fa3 backend is sm_90 only)


def _flashinfer():
    os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", _FI_BASE)
    # the CUDA build of flashinfer's norm kernels: the one the reference's
    # RSMNormWithoutResidual calls (src/layers/rsm_norm.cu:29,49)
    os.environ.setdefault("FLASHINFER_USE_CUDA_NORM", "1")
    import flashinfer

    return flashinfer


def prebuild(head_dims=(64, 128, 256), dtype=torch.bfloat16) -> None:
    """Compile flashinfer's paged-decode kernels, and the norm and rotary
    kernels the fused Q/K norm + store is checked against, for sm_100a into
    the package's build folder (no GPU needed)."""
    os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", _FI_BASE)
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0")
    os.environ.setdefault("FLASHINFER_USE_CUDA_NORM", "1")
    from flashinfer.decode import get_batch_decode_module
    from flashinfer.norm import get_norm_module
    from flashinfer.prefill import get_batch_prefill_module
    from flashinfer.rope import get_rope_module

    for d in head_dims:
        get_batch_decode_module(dtype, dtype, dtype, torch.int32, d, d, 0, False, False)
    get_batch_prefill_module(PREFILL_BACKEND, dtype, dtype, dtype, torch.int32, 128, 128, 0, False, False, False)
    get_norm_module()
    get_rope_module()


class PagedDecodeAttention:
    """Decode attention over the paged pool (one new token per sequence).

    q: [B, num_qo_heads, head_dim]; k, v: [B, num_kv_heads, head_dim];
    k_pages, v_pages: one layer's pool views [num_pages, page_size,
    num_kv_heads, head_dim] (MHAKVCache.KCache(layer) / VCache(layer)).
    """

    def __init__(self, num_qo_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
                 device: torch.device | str = "cuda", workspace_bytes: int = 128 << 20):
        fi = _flashinfer()
        self.num_qo_heads, self.num_kv_heads, self.head_dim, self.page_size = (num_qo_heads, num_kv_heads, head_dim,
                                                                                page_size)
        self.workspace = torch.empty(workspace_bytes, dtype=torch.uint8, device=device)
        self.wrapper = fi.BatchDecodeWithPagedKVCacheWrapper(self.workspace, "NHD")
        self.slots = None

    def plan(self, index: BatchIndex, dtype: torch.dtype = torch.bfloat16) -> None:
        """Once per step, after the index build: hand the page arrays to flashinfer."""
        self.wrapper.plan(index.kv_indptr, index.kv_indices, index.kv_last_page_len, self.num_qo_heads,
                          self.num_kv_heads, self.head_dim, self.page_size, q_data_type=dtype, kv_data_type=dtype)
        self.slots = index.slot_mapping

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_pages: torch.Tensor,
                v_pages: torch.Tensor) -> torch.Tensor:
        """One layer: store this step's K/V rows, then attend over the pool."""
        P, ps, H, D = k_pages.shape
        n = k.shape[0]
        store_kv_cache(k.reshape(n, H * D), v.reshape(n, H * D), k_pages.view(P * ps, H * D),
                       v_pages.view(P * ps, H * D), self.slots)
        return self.wrapper.run(q, (k_pages, v_pages))


class PagedPrefillAttention:
    """Causal attention of each sequence's new tokens over its whole paged
    history, new tokens included (query t of sequence i sits at position
    prior_len_i + t).  q: [N, num_qo_heads, head_dim] ragged by qo_indptr;
    k, v: [N, num_kv_heads, head_dim]; pool views as for decode."""

    def __init__(self, num_qo_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
                 device: torch.device | str = "cuda", workspace_bytes: int = 256 << 20):
        fi = _flashinfer()
        self.num_qo_heads, self.num_kv_heads, self.head_dim, self.page_size = (num_qo_heads, num_kv_heads, head_dim,
                                                                                page_size)
        self.workspace = torch.empty(workspace_bytes, dtype=torch.uint8, device=device)
        self.wrapper = fi.BatchPrefillWithPagedKVCacheWrapper(self.workspace, "NHD", backend=PREFILL_BACKEND)
        self.slots = None

    def plan(self, index: BatchIndex, dtype: torch.dtype = torch.bfloat16) -> None:
        self.wrapper.plan(index.qo_indptr, index.kv_indptr, index.kv_indices, index.kv_last_page_len,
                          self.num_qo_heads, self.num_kv_heads, self.head_dim, self.page_size, causal=True,
                          q_data_type=dtype, kv_data_type=dtype)
        self.slots = index.slot_mapping

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_pages: torch.Tensor,
                v_pages: torch.Tensor) -> torch.Tensor:
        P, ps, H, D = k_pages.shape
        n = k.shape[0]
        store_kv_cache(k.reshape(n, H * D), v.reshape(n, H * D), k_pages.view(P * ps, H * D),
                       v_pages.view(P * ps, H * D), self.slots)
        return self.wrapper.run(q, (k_pages, v_pages))


def paged_decode_reference(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor, index: BatchIndex,
                           page_size: int) -> torch.Tensor:
    """Plain-torch fp32 paged decode attention that reads the pool only
    through the page arrays (kv_indptr, kv_indices, kv_last_page_len)."""
    B, Hq, D = q.shape
    Hk = k_pages.shape[2]
    indptr = index.kv_indptr.tolist()
    indices = index.kv_indices
    last = index.kv_last_page_len.tolist()
    out = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    for i in range(B):
        pages = indices[indptr[i]:indptr[i + 1]].long()
        n = (len(pages) - 1) * page_size + last[i]
        k = k_pages[pages].reshape(-1, Hk, D)[:n].float()
        v = v_pages[pages].reshape(-1, Hk, D)[:n].float()
        k = k.repeat_interleave(Hq // Hk, dim=1)
        v = v.repeat_interleave(Hq // Hk, dim=1)
        s = torch.einsum("hd,nhd->hn", q[i].float(), k) / D ** 0.5
        out[i] = torch.einsum("hn,nhd->hd", torch.softmax(s, dim=-1), v)
    return out
