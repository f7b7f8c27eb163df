"""The C++ libtorch front end on the GPU: the reference's MHAKVCache tests
(test/mha_kvcache_test.cpp:260-575), seeded, at page sizes 1 and 16, plus the
batch manager's per-step index driver checked against the CPU oracle."""
import numpy as np
import pytest
import torch

import yllang_b200 as yl
from _kvutil import assert_index_equal
from oracle import kvpath as orc

pytestmark = pytest.mark.gpu
C = yl.load_extension()
LAYER_FIRST = C.KVCacheLayout.kLayerFirst
PAGE_FIRST = C.KVCacheLayout.kPageFirst


@pytest.mark.parametrize("page_size", [1, 16])
def test_store_kv_stores_correctly(cuda, page_size):  # TestStoreKVStoresCorrectly (:260-333)
    torch.manual_seed(0)
    H, D, P = 8, 64, 8
    cache = C.MHAKVCache(2, P, H, D, LAYER_FIRST, "cuda", torch.float32, page_size)
    k = torch.randn(2, 3, H, D, device=cuda)
    v = torch.randn(2, 3, H, D, device=cuda)
    loc = torch.randperm(6 * page_size, device=cuda)[:6]
    cache.StoreKV(k, v, loc, 0)
    kc = cache.KCache(0).reshape(P * page_size, H, D)
    vc = cache.VCache(0).reshape(P * page_size, H, D)
    for i, s in enumerate(loc.tolist()):
        assert torch.equal(kc[s], k.view(6, H, D)[i]) and torch.equal(vc[s], v.view(6, H, D)[i])
    assert float(cache.KCache(1).abs().sum()) == 0.0


def test_store_kv_overwrites_same_page(cuda):  # TestStoreKVOverwritesSamePage (:338-393)
    cache = C.MHAKVCache(2, 8, 8, 64, PAGE_FIRST, "cuda", torch.float32, 1)
    loc = torch.full((1,), 1, dtype=torch.int64, device=cuda)
    k1, v1, k2, v2 = (torch.randn(1, 1, 8, 64, device=cuda) for _ in range(4))
    cache.StoreKV(k1, v1, loc, 0)
    cache.StoreKV(k2, v2, loc, 0)
    assert torch.equal(cache.KCache(0)[1, 0], k2[0, 0]) and torch.equal(cache.VCache(0)[1, 0], v2[0, 0])


def test_store_kv_with_empty_input(cuda):  # TestStoreKVWithEmptyInput (:398-435)
    cache = C.MHAKVCache(2, 8, 8, 64, PAGE_FIRST, "cuda", torch.float32, 1)
    e = torch.randn(0, 3, 8, 64, device=cuda)
    cache.StoreKV(e, e, torch.zeros(0, dtype=torch.int64, device=cuda), 0)
    e = torch.randn(2, 0, 8, 64, device=cuda)
    cache.StoreKV(e, e, torch.zeros(0, dtype=torch.int64, device=cuda), 0)
    torch.cuda.synchronize()
    assert float(cache.Buffer().abs().sum()) == 0.0


def test_store_kv_multiple_random_writes(cuda):  # TestStoreKVMultipleRandomWrites (:473-575), seeded
    g = torch.Generator().manual_seed(7)
    P, H, D = 128, 8, 64
    cache = C.MHAKVCache(100, P, H, D, PAGE_FIRST, "cuda", torch.float32, 1)
    last = {}
    for _ in range(2000):
        b = int(torch.randint(1, 4, (1,), generator=g))
        s = int(torch.randint(1, 5, (1,), generator=g))
        k = torch.randn(b, s, H, D, generator=g)
        v = torch.randn(b, s, H, D, generator=g)
        loc = torch.randperm(b * s, generator=g)
        for i, p in enumerate(loc.tolist()):
            last[p] = (k.view(-1, H, D)[i], v.view(-1, H, D)[i])
        cache.StoreKV(k.to(cuda), v.to(cuda), loc.to(cuda), 0)
    kc, vc = cache.KCache(0).cpu(), cache.VCache(0).cpu()
    for p, (kk, vv) in last.items():
        assert torch.equal(kc[p, 0], kk) and torch.equal(vc[p, 0], vv)


def test_store_all_layers_matches_per_layer(cuda):
    torch.manual_seed(1)
    L, P, ps, H, D, N = 4, 32, 16, 2, 128, 70
    a = C.MHAKVCache(L, P, H, D, LAYER_FIRST, "cuda", torch.bfloat16, ps)
    b = C.MHAKVCache(L, P, H, D, LAYER_FIRST, "cuda", torch.bfloat16, ps)
    k = torch.randn(L, N, H, D, device=cuda).to(torch.bfloat16)
    v = torch.randn(L, N, H, D, device=cuda).to(torch.bfloat16)
    loc = torch.randperm(P * ps, device=cuda)[:N].to(torch.int32)
    a.StoreKVAllLayers(k, v, loc)
    for layer in range(L):
        b.StoreKV(k[layer], v[layer], loc, layer)
    torch.cuda.synchronize()
    assert torch.equal(a.Buffer().view(torch.int16), b.Buffer().view(torch.int16))


def test_reference_signature_checks_row_size(cuda):
    k = torch.randn(3, 512, device=cuda)  # 2048-byte rows
    kc = torch.zeros(16, 512, device=cuda)
    vc = torch.zeros_like(kc)
    idx = torch.tensor([3, 0, 9], device=cuda)
    C.StoreKVCache2048(k, k, kc, vc, idx)
    torch.cuda.synchronize()
    assert torch.equal(kc[idx], k)
    with pytest.raises(C.PanicError):
        C.StoreKVCache2048(k[:, :256], k[:, :256], kc[:, :256], vc[:, :256], idx)


def _oracle_for(requests, manager, page_size):
    host = manager.HostPageTable().numpy()
    prior = [r.cached_len for r in requests]
    new = [r.device_len - r.cached_len for r in requests]
    rows = [r.table_index for r in requests]
    return orc.build_index(prior, new, host, page_size, table_index=rows, num_pages=manager.NumPages())


def test_batch_manager_steps_match_oracle(cuda):
    """Prefill four requests, then decode three steps; every batch's arrays
    match the oracle on the manager's own page table, and stores through
    MHAKVCache land on the slots the batch names."""
    ps, P = 16, 512
    manager = C.KVCacheManager(P, 16, 64, ps, "cuda")
    bm = C.BatchManager(manager)
    cache = C.MHAKVCache(2, P, 8, 128, LAYER_FIRST, "cuda", torch.bfloat16, ps)
    rows = [manager.AllocateTableSlot() for _ in range(4)]
    lens = [30, 50, 7, 100]
    reqs = [C.RequestSlot(r, 0, n) for r, n in zip(rows, lens)]
    for step in range(4):
        batch = bm.NextBatch(reqs)
        want = _oracle_for(reqs, manager, ps)
        got = {n: getattr(batch.index, n).cpu().numpy() for n in
               ("kv_indptr", "kv_indices", "kv_last_page_len", "qo_indptr", "slot_mapping")}
        assert want["err"] == 0
        assert_index_equal(got, want)
        N = batch.num_tokens
        k = torch.randn(N, 8, 128, device=cuda).to(torch.bfloat16)
        for layer in range(2):
            cache.StoreKV(k, k, batch.out_loc, layer)
        kc = cache.KCache(1).reshape(P * ps, 8, 128)
        assert torch.equal(kc[batch.out_loc.long()].view(torch.int16), k.view(torch.int16))
        reqs = [C.RequestSlot(r.table_index, r.device_len, r.device_len + 1) for r in reqs]  # one decode token
    used = manager.HostPageTable()
    assert (used[rows] >= 0).sum() == sum(-(-(n + 3) // ps) for n in lens)
    for r in rows:
        manager.Release(r)
    assert manager.RemainingPageCount() == P and manager.RemainingTableSlots() == 16


def test_build_batch_index_binding(cuda):
    rng = np.random.default_rng(0)
    prior = rng.integers(0, 300, 40).astype(np.int32)
    new = rng.integers(0, 20, 40).astype(np.int32)
    table = rng.integers(0, 1 << 16, (40, 24)).astype(np.int32)
    t = lambda a: torch.from_numpy(a).to(cuda)
    out = C.BuildBatchIndex(t(prior), t(new), t(table), 16, None, 1 << 16)
    want = orc.build_index(prior, new, table, 16, num_pages=1 << 16)
    got = {n: getattr(out, n).cpu().numpy() for n in
           ("kv_indptr", "kv_indices", "kv_last_page_len", "qo_indptr", "slot_mapping")}
    assert_index_equal(got, want)
