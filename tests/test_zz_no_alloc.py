"""The allocation-free decode attention entry point
(yl_paged_decode_attention_noalloc, include/yl_attention.h), for callers that
must not allocate device memory on their hot path — an engine that reserves
all of its device memory at start-up, or host code running under another
framework's caching allocator it cannot reach.  Called through the C ABI
twice in a row on the same step, its output must match the planned decode
path of the C++ Attention layer (which plans into a workspace it allocates)
within the attention tests' tolerance (2e-2 absolute + 2e-2 relative, bf16),
and the two calls must agree exactly: each call rewrites the work lists the
calls share.  Collected last, so a run that stops at its first failure has
run every other test before this one."""
import ctypes
import os

import numpy as np
import pytest
import torch

import yllang_b200 as yl

pytestmark = pytest.mark.gpu
ATOL = RTOL = 2e-2
LIB = os.path.join(os.path.dirname(os.path.abspath(yl.__file__)), "libyl_attention.so")
MAX_BATCH = 16384
YL_ERR_BAD_SIZE = -2


class DecodeArgs(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("o", ctypes.c_void_p), ("k_cache", ctypes.c_void_p),
                ("v_cache", ctypes.c_void_p), ("kv_indptr", ctypes.c_void_p), ("kv_indices", ctypes.c_void_p),
                ("kv_last_page_len", ctypes.c_void_p), ("q_row_stride", ctypes.c_int64),
                ("q_head_stride", ctypes.c_int64), ("page_stride", ctypes.c_int64), ("slot_stride", ctypes.c_int64),
                ("head_stride", ctypes.c_int64), ("batch_size", ctypes.c_int32), ("num_qo_heads", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("page_size", ctypes.c_int32),
                ("dtype", ctypes.c_int32), ("sm_scale", ctypes.c_float)]


def _entry():
    f = ctypes.CDLL(LIB).yl_paged_decode_attention_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.POINTER(DecodeArgs), ctypes.c_void_p]
    return f


def test_no_alloc_decode_matches_the_planned_path_on_two_calls(cuda):
    C = yl.load_extension()
    Hq, Hk, D, ps, P, B = 32, 8, 128, 16, 2048, 24
    rng = np.random.default_rng(11)
    prior = rng.integers(20, 400, B).astype(np.int32)
    g = torch.Generator(device=cuda).manual_seed(4)
    W = int((prior.max() + 1 + ps - 1) // ps)
    table = torch.randperm(P, generator=torch.Generator().manual_seed(5))[:B * W].to(torch.int32).view(B, W).to(cuda)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    cache = C.MHAKVCache(1, P, Hk, D, C.KVCacheLayout.kLayerFirst, "cuda", torch.bfloat16, ps)
    n_hist = int(prior.sum())
    hist_k = torch.randn(n_hist, Hk, D, generator=g, device=cuda).to(torch.bfloat16)
    hist_v = torch.randn(n_hist, Hk, D, generator=g, device=cuda).to(torch.bfloat16)
    pre = C.BuildBatchIndex(t(np.zeros(B)), t(prior), table, ps, num_pages=P)
    cache.StoreKV(hist_k, hist_v, pre.slot_mapping, 0)
    idx = C.BuildBatchIndex(t(prior), t(np.ones(B)), table, ps, num_pages=P)
    qkv = torch.randn(B, (Hq + 2 * Hk) * D, generator=g, device=cuda).to(torch.bfloat16)

    # the existing entry point: the planned decode of the C++ layer (stores the step's K/V too)
    ctx = C.AttentionContext("cuda")
    ctx.Plan(idx, Hq, Hk, D, ps, torch.bfloat16)
    want = C.Attention(0, Hq, Hk, D, cache).Forward(qkv, ctx).view(B, Hq, D)

    q = qkv[:, :Hq * D].unflatten(1, (Hq, D))  # strided rows of the projection output
    kc, vc = cache.KCache(0), cache.VCache(0)  # [P, ps, Hk, D]
    f = _entry()
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for _ in range(2):
        o = torch.full((B, Hq, D), float("nan"), dtype=torch.bfloat16, device=cuda)
        a = DecodeArgs(q=q.data_ptr(), o=o.data_ptr(), k_cache=kc.data_ptr(), v_cache=vc.data_ptr(),
                       kv_indptr=idx.kv_indptr.data_ptr(), kv_indices=idx.kv_indices.data_ptr(),
                       kv_last_page_len=idx.kv_last_page_len.data_ptr(), q_row_stride=q.stride(0),
                       q_head_stride=q.stride(1), page_stride=kc.stride(0), slot_stride=kc.stride(1),
                       head_stride=kc.stride(2), batch_size=B, num_qo_heads=Hq, num_kv_heads=Hk, head_dim=D,
                       page_size=ps, dtype=0, sm_scale=1.0 / D ** 0.5)
        assert f(ctypes.byref(a), stream) == 0
        outs.append(o)
    torch.cuda.synchronize()
    for o in outs:
        torch.testing.assert_close(o.float(), want.float(), atol=ATOL, rtol=RTOL)
    assert torch.equal(outs[0], outs[1])


def test_no_alloc_decode_refuses_batches_beyond_its_scratch(cuda):
    a = DecodeArgs(batch_size=MAX_BATCH + 1, num_qo_heads=8, num_kv_heads=8, head_dim=128, page_size=16)
    assert _entry()(ctypes.byref(a), None) == YL_ERR_BAD_SIZE
