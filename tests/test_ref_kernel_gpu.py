"""The B200 store vs the reference's own store kernel, run on the same GPU.

oracle/_ref/libref_store.so is the reference's StoreKVCache launcher and
StoreKVCacheKernel (src/kvcache/store_kv_cache.cu:46-163) compiled from the
reference sources for sm_100a (oracle/Makefile, target `ref`).  Both stores
start from identical sentinel-filled pools and must leave them byte-identical;
the CPU oracle must agree with both, which pins the oracle to the reference.
The reference accepts rows of 512/1024/2048/4096 bytes and reads int64 slots
only (store_kv_cache.cu:127, src/include/cuda/memory.cuh:151).
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import yllang_b200 as yl
from _kvutil import host_bytes, oracle_store
from yllang_b200 import workloads

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_STORE = os.path.join(ROOT, "oracle", "_ref", "libref_store.so")
DTYPE_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


@pytest.fixture(scope="module")
def ref_store():
    assert os.path.exists(REF_STORE), "reference harness not built (make -C oracle ref)"
    L = ctypes.CDLL(REF_STORE)
    f = L.ref_store_kv_cache
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int] + [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 4
    return f


def _ref_call(f, k, v, kc, vc, slots):
    rc = f(k.shape[1] * k.element_size(), DTYPE_CODE[k.dtype], k.device.index or 0, k.data_ptr(), v.data_ptr(),
           kc.data_ptr(), vc.data_ptr(), slots.data_ptr(), k.shape[0], k.stride(0), kc.shape[0], kc.stride(0))
    assert rc == 0, rc


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("row_bytes", [512, 1024, 2048, 4096])
def test_store_matches_reference_kernel(cuda, ref_store, dtype, row_bytes):
    item = torch.tensor([], dtype=dtype).element_size()
    E = row_bytes // item
    N, S = 301, 4096
    torch.manual_seed(row_bytes)
    k = torch.randn(N, E).to(dtype).to(cuda)
    v = torch.randn(N, E).to(dtype).to(cuda)
    init = torch.randn(2, S, E).to(dtype).to(cuda)
    slots = torch.randperm(S)[:N].to(cuda)
    kc_ref, vc_ref = init[0].clone(), init[1].clone()
    kc, vc = init[0].clone(), init[1].clone()
    want_k, want_v, _ = oracle_store(k, v, kc, vc, slots)
    _ref_call(ref_store, k, v, kc_ref, vc_ref, slots)
    yl.store_kv_cache(k, v, kc, vc, slots)
    torch.cuda.synchronize()
    assert np.array_equal(host_bytes(kc), host_bytes(kc_ref))
    assert np.array_equal(host_bytes(vc), host_bytes(vc_ref))
    assert np.array_equal(host_bytes(kc_ref), want_k) and np.array_equal(host_bytes(vc_ref), want_v)


def test_step_matches_reference_kernel(cuda, ref_store):
    """Decode-shaped step: slots from the index build, every layer stored by both kernels."""
    b = workloads.llama3_decode(num_pages=2048, batch=64, layers=4, ctx_hi=2048)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    idx = yl.build_index(t(b.prior_len), t(b.new_len), t(b.page_table), b.page_size, num_pages=b.num_pages,
                         kv_indices_capacity=b.total_pages, slot_capacity=b.tokens)
    E = b.kv_heads * b.head_dim
    S = b.num_pages * b.page_size
    torch.manual_seed(0)
    pool = torch.randn(2, b.layers, S, E).to(torch.bfloat16).to(cuda)
    pool_ref = pool.clone()
    k = torch.randn(b.layers, b.tokens, E).to(torch.bfloat16).to(cuda)
    v = torch.randn(b.layers, b.tokens, E).to(torch.bfloat16).to(cuda)
    yl.store_kv_cache(k, v, pool[0], pool[1], idx.slot_mapping)  # all layers, one launch
    for layer in range(b.layers):  # the reference: one launch per layer
        _ref_call(ref_store, k[layer], v[layer], pool_ref[0, layer], pool_ref[1, layer], idx.slot_mapping)
    torch.cuda.synchronize()
    assert torch.equal(pool.view(torch.int16), pool_ref.view(torch.int16))
