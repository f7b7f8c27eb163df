"""The C++ libtorch front end (yllang_b200._C) on the host: page allocator,
page table, pool views and contract checks.  No GPU needed.

Construction and view tests port TestConstructorCreatesCorrectShape*,
TestKCacheAndVCacheAreIndependent and TestNumLayersAndDevice of the
reference's test/mha_kvcache_test.cpp (:27-192, :440-468)."""
import pytest
import torch

import yllang_b200 as yl

C = yl.load_extension()


@pytest.fixture(autouse=True)
def single_rank():
    C.SetDistributedInfo(0, 1)
    yield
    C.SetDistributedInfo(0, 1)


@pytest.mark.parametrize("layout", [C.KVCacheLayout.kPageFirst, C.KVCacheLayout.kLayerFirst])
@pytest.mark.parametrize("page_size", [1, 16])
def test_pool_views_have_reference_shape(layout, page_size):
    cache = C.MHAKVCache(2, 4, 8, 64, layout, "cpu", torch.float32, page_size)
    for layer in range(2):
        k, v = cache.KCache(layer), cache.VCache(layer)
        assert tuple(k.shape) == (4, page_size, 8, 64) and tuple(v.shape) == (4, page_size, 8, 64)
        assert k.data_ptr() != v.data_ptr()
        assert k.dtype == torch.float32 and k.device.type == "cpu"
    assert cache.KCache(0).data_ptr() != cache.KCache(1).data_ptr()
    assert cache.NumLayers() == 2 and cache.Device() == "cpu"
    assert cache.NumSlots() == 4 * page_size
    assert float(cache.Buffer().abs().sum()) == 0.0  # zero-filled like the reference (mha_kvcache.h:50,53)


def test_tensor_parallel_head_split():
    C.SetDistributedInfo(1, 4)
    cache = C.MHAKVCache(1, 4, 8, 128, C.KVCacheLayout.kLayerFirst, "cpu", torch.bfloat16, 16)
    assert cache.NumLocalKVHeads() == 2 and tuple(cache.KCache(0).shape) == (4, 16, 2, 128)
    C.SetDistributedInfo(0, 3)
    with pytest.raises(C.PanicError):
        C.MHAKVCache(1, 4, 8, 128, C.KVCacheLayout.kLayerFirst, "cpu", torch.bfloat16, 16)


def test_store_requires_cuda_tensors():
    cache = C.MHAKVCache(1, 8, 8, 64, C.KVCacheLayout.kLayerFirst, "cpu", torch.float32, 1)
    k = torch.zeros(2, 8, 64)
    with pytest.raises(C.PanicError, match="CUDA"):
        cache.StoreKV(k, k, torch.arange(2), 0)
    with pytest.raises(C.PanicError):
        C.StoreKVCache2048(torch.zeros(2, 100), torch.zeros(2, 100), torch.zeros(8, 100), torch.zeros(8, 100),
                           torch.arange(2))
    cache.StoreKV(torch.zeros(0, 8, 64), torch.zeros(0, 8, 64), torch.zeros(0, dtype=torch.int64), 0)  # no-op


def test_page_allocator_hands_out_each_page_once():
    m = C.KVCacheManager(100, 4, 16, 16, "cpu")
    a = m.AllocatePages(60)
    b = m.AllocatePages(40)
    ids = torch.cat([a, b]).tolist()
    assert sorted(ids) == list(range(100))  # exactly pages 0..P-1, no duplicates
    assert m.RemainingPageCount() == 0
    with pytest.raises(RuntimeError, match="not enough pages"):
        m.AllocatePages(1)
    m.FreePages(a[:10])
    assert m.RemainingPageCount() == 10
    with pytest.raises(RuntimeError):
        m.FreePages(torch.tensor([100], dtype=torch.int32))


def test_table_rows_reserve_release_sync():
    m = C.KVCacheManager(64, 3, 8, 16, "cpu")
    rows = [m.AllocateTableSlot() for _ in range(3)]
    assert sorted(rows) == [0, 1, 2] and m.RemainingTableSlots() == 0
    with pytest.raises(RuntimeError, match="table slots"):
        m.AllocateTableSlot()
    assert m.Reserve(rows[0], 33).numel() == 3 and m.PagesInRow(rows[0]) == 3
    assert m.Reserve(rows[0], 40).numel() == 0  # still 3 pages
    assert m.Reserve(rows[0], 49).numel() == 1
    m.Reserve(rows[1], 16)
    with pytest.raises(RuntimeError, match="more pages than a page-table row"):
        m.Reserve(rows[2], 16 * 8 + 1)
    m.SyncPageTable()
    assert torch.equal(m.PageTable(), m.HostPageTable())
    host = m.HostPageTable()
    used = host[host >= 0].tolist()
    assert len(used) == len(set(used)) == 5
    m.Release(rows[0])
    m.SyncPageTable()
    assert torch.equal(m.PageTable(), m.HostPageTable())
    assert (m.HostPageTable()[rows[0]] == -1).all() and m.RemainingPageCount() == 64 - 1
    assert m.RemainingTableSlots() == 1


def test_device_page_pool_rejects_bad_arguments():
    with pytest.raises(C.PanicError, match="CUDA device"):
        C.DevicePagePool(16, "cpu")
    with pytest.raises(C.PanicError, match="num_pages"):
        C.DevicePagePool(0, "cpu")


def test_qk_norm_rope_options_defaults():
    o = C.QKNormRope()
    assert o.q_weight is None and o.k_weight is None and o.cos_sin_cache is None and o.positions is None
    assert o.eps == pytest.approx(1e-6) and o.interleaved is False
    o.eps, o.interleaved = 1e-5, True
    assert o.eps == pytest.approx(1e-5) and o.interleaved is True


def test_qk_norm_rope_store_kv_checks_before_any_launch():
    """Shape and dtype contract first, then the device: CPU tensors are refused
    (no host fallback)."""
    q = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    k = torch.zeros(4, 1, 128, dtype=torch.bfloat16)
    kc = torch.zeros(8, 128, dtype=torch.bfloat16)
    idx = torch.zeros(4, dtype=torch.int64)
    with pytest.raises(C.PanicError, match="bf16 or fp16"):
        C.QKNormRopeStoreKV(q.float(), k.float(), k.float(), kc.float(), kc.float(), idx, C.QKNormRope(), q.float())
    with pytest.raises(C.PanicError, match="shapes"):
        C.QKNormRopeStoreKV(q, k, k, kc, kc, idx, C.QKNormRope(), q[:3])
    with pytest.raises(C.PanicError, match="contiguous heads"):
        C.QKNormRopeStoreKV(q.transpose(1, 2), k, k, kc, kc, idx, C.QKNormRope(), q)
    with pytest.raises(C.PanicError, match="CUDA tensors"):
        C.QKNormRopeStoreKV(q, k, k, kc, kc, idx, C.QKNormRope(), q)


def test_index_front_end_checks_before_any_launch():
    w = torch.zeros(10, 64, dtype=torch.bfloat16)
    with pytest.raises(C.PanicError, match="weights"):
        C.Index(torch.zeros(3, dtype=torch.int32), w.t(), torch.zeros(3, 10, dtype=torch.bfloat16))
    with pytest.raises(C.PanicError, match="destination"):
        C.Index(torch.zeros(3, dtype=torch.int32), w, torch.zeros(3, 32, dtype=torch.bfloat16))
    with pytest.raises(C.PanicError, match="CUDA tensors"):
        C.Index(torch.zeros(3, dtype=torch.int32), w, torch.zeros(3, 64, dtype=torch.bfloat16))


def test_make_2d_indices_front_end_checks_before_any_launch():
    r = [torch.tensor([0, 1, 3])]
    with pytest.raises(C.PanicError, match="2-D"):
        C.Make2DIndices(torch.zeros(4), r)
    with pytest.raises(C.PanicError, match="CUDA"):
        C.Make2DIndices(torch.zeros(4, 8), r)
