"""Device page allocator (yl_reserve_pages / yl_release_pages) on the GPU,
bit-exact against the oracle's restatement of KVCacheManager's free list
(src/include/kvcache/cache_manager.h:105-155): seeded multi-step reserve /
release sequences (page sizes 1 and 16, batches beyond one 1024-thread chunk,
permuted table rows), the all-or-nothing error cases, the index build on the
table the device filled, a CUDA graph of reserve + index build replayed with
no host round trip, and the C++ front end against the host KVCacheManager."""
import numpy as np
import pytest
import torch

import yllang_b200 as yl
from _kvutil import assert_index_equal, index_outputs
from oracle import kvpath as orc

pytestmark = pytest.mark.gpu


def _state(pool: yl.DevicePagePool, table: torch.Tensor):
    torch.cuda.synchronize()
    return pool.free_list().cpu().numpy(), table.cpu().numpy()


@pytest.mark.parametrize("ps,B", [(1, 40), (16, 200), (16, 2500)])
def test_reserve_release_sequence_matches_oracle(cuda, ps, B):
    rng = np.random.default_rng(B + ps)
    W = 96
    P = B * W // 2
    rows = rng.permutation(B + 7)[:B].astype(np.int32)  # sequence i lives in row rows[i]
    table = torch.full((B + 7, W), -1, dtype=torch.int32, device=cuda)
    otable = np.full((B + 7, W), -1, np.int32)
    pool, opool = yl.DevicePagePool(P, cuda), orc.PagePool(P)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    lens = np.zeros(B, np.int64)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    for step in range(12):
        if step % 4 == 3:
            done = rng.choice(B, size=max(1, B // 5), replace=False)
            pool.release(table, t(rows[done]), t(lens[done]), ps, error_word=err)
            assert opool.release(otable, rows[done], lens[done], ps) == 0
            lens[done] = 0
        else:
            new = np.minimum(rng.integers(0, 2 * ps + 3, B), W * ps - lens)
            pool.reserve(table, t(lens), t(new), ps, table_index=t(rows), error_word=err)
            assert opool.reserve(otable, lens, new, ps, table_index=rows) == 0
            lens += new
        free, got = _state(pool, table)
        assert int(err.item()) == 0
        assert np.array_equal(free, opool.free_list()), step
        assert np.array_equal(got, otable), step


def test_reserve_release_errors_change_nothing(cuda):
    P, W, ps = 10, 8, 4
    t = lambda a: torch.tensor(a, dtype=torch.int32, device=cuda)
    pool = yl.DevicePagePool(P, cuda)
    table = torch.full((3, W), -1, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for prior, new, rows, bit in [([0, 0], [16, 30], None, yl.DEVERR_POOL_EMPTY),
                                  ([0, 0], [16, 33], None, 0x4),
                                  ([0, -1], [4, 4], None, 0x20),
                                  ([0, 0], [4, 4], [0, 3], 0x80)]:
        err.zero_()
        pool.reserve(table, t(prior), t(new), ps, table_index=None if rows is None else t(rows), error_word=err)
        free, got = _state(pool, table)
        assert int(err.item()) == bit
        assert (got == -1).all() and free.tolist() == list(range(P))
    pool.reserve(table, t([0, 0]), t([8, 4]), ps, error_word=err)
    free, got = _state(pool, table)
    assert got[0, :2].tolist() == [8, 9] and got[1, :1].tolist() == [7] and free.tolist() == list(range(7))
    before = table.cpu().numpy()
    err.zero_()
    pool.reserve(table, t([0, 0]), t([4, 4]), ps, table_index=t([2, 2]), error_word=err)  # row 2 twice
    free, got = _state(pool, table)
    assert int(err.item()) == yl.DEVERR_DUPLICATE_ROW and free.tolist() == list(range(7))
    assert np.array_equal(got, before)
    err.zero_()
    pool.release(table, t([0, 0]), t([8, 8]), ps, error_word=err)  # row 0's pages would enter the list twice
    free, got = _state(pool, table)
    assert int(err.item()) == yl.DEVERR_DUPLICATE_ROW and free.tolist() == list(range(7))
    assert np.array_equal(got, before)
    full = yl.DevicePagePool(P, cuda, free_pages=torch.arange(9, dtype=torch.int32))
    err.zero_()
    full.release(table, t([0]), t([8]), ps, error_word=err)  # 9 + 2 > 10
    free, got = _state(full, table)
    assert int(err.item()) == yl.DEVERR_POOL_OVERFLOW and free.tolist() == list(range(9))
    assert np.array_equal(got, before)
    pool.release(table, t([0, 1]), t([8, 4]), ps)
    free, got = _state(pool, table)
    assert free.tolist() == list(range(7)) + [8, 9, 7] and (got == -1).all()
    # a corrupt table entry: nothing moves
    bad = torch.tensor([[5, 11] + [-1] * (W - 2)], dtype=torch.int32, device=cuda)
    small = yl.DevicePagePool(P, cuda, free_pages=torch.arange(6, dtype=torch.int32))
    err.zero_()
    small.release(bad, t([0]), t([8]), ps, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == yl.DEVERR_PAGE_RANGE and small.free_count() == 6


@pytest.mark.parametrize("case", ["reserve", "release"])
@pytest.mark.parametrize("spread", [False, True])
def test_duplicate_rows_change_nothing(cuda, case, spread):
    """A table row named twice in one call (batches over several 1024-thread
    chunks; rows within one bitmap window, or spread over a 700,000-row table
    so the check walks several windows) sets DEVERR_DUPLICATE_ROW and leaves
    the free list and the table as they were; the same batch without the
    repeat goes through, as in the oracle."""
    rng = np.random.default_rng(11 + int(spread))
    B, ps, W = 2500, 16, 4
    R = 700_000 if spread else B + 50
    P = 4 * B + 100
    rows = (np.sort(rng.choice(R, size=B, replace=False)) if spread else rng.permutation(R)[:B]).astype(np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    table = torch.full((R, W), -1, dtype=torch.int32, device=cuda)
    otable = np.full((R, W), -1, np.int32)
    pool, opool = yl.DevicePagePool(P, cuda), orc.PagePool(P)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    zeros = np.zeros(B, np.int32)
    lens = rng.integers(1, W * ps + 1, B).astype(np.int32)
    if case == "release":  # fill the rows first
        pool.reserve(table, t(zeros), t(lens), ps, table_index=t(rows), error_word=err)
        assert opool.reserve(otable, zeros, lens, ps, table_index=rows) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    dup, dlens = rows.copy(), lens.copy()
    dup[B - 3], dlens[B - 3] = dup[5], lens[5]  # far apart: first and last windows when spread
    free0, table0 = _state(pool, table)
    if case == "reserve":
        pool.reserve(table, t(zeros), t(lens), ps, table_index=t(dup), error_word=err)
        want = opool.reserve(otable, zeros, lens, ps, table_index=dup)
    else:  # the repeated row releases the tokens it holds: nothing but the repeat is wrong
        pool.release(table, t(dup), t(dlens), ps, error_word=err)
        want = opool.release(otable, dup, dlens, ps)
    free, got = _state(pool, table)
    assert want == yl.DEVERR_DUPLICATE_ROW and int(err.item()) == want
    assert np.array_equal(free, free0) and np.array_equal(got, table0)
    err.zero_()
    if case == "reserve":
        pool.reserve(table, t(zeros), t(lens), ps, table_index=t(rows), error_word=err)
        assert opool.reserve(otable, zeros, lens, ps, table_index=rows) == 0
    else:
        pool.release(table, t(rows), t(lens), ps, error_word=err)
        assert opool.release(otable, rows, lens, ps) == 0
    free, got = _state(pool, table)
    assert int(err.item()) == 0
    assert np.array_equal(free, opool.free_list()) and np.array_equal(got, otable)


def test_index_build_on_device_reserved_table(cuda):
    """Reserve then build the batch index from the same device lengths: the
    page ids the index reads never leave the device."""
    rng = np.random.default_rng(4)
    B, W, ps, P = 300, 64, 16, 20000
    prior = rng.integers(0, 400, B).astype(np.int32)
    new = rng.integers(1, 40, B).astype(np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    pool, opool = yl.DevicePagePool(P, cuda), orc.PagePool(P)
    table = torch.full((B, W), -1, dtype=torch.int32, device=cuda)
    otable = np.full((B, W), -1, np.int32)
    zeros = np.zeros(B, np.int32)
    pool.reserve(table, t(zeros), t(prior), ps)  # the history
    assert opool.reserve(otable, zeros, prior, ps) == 0
    pool.reserve(table, t(prior), t(new), ps)  # this step
    assert opool.reserve(otable, prior, new, ps) == 0
    idx = yl.build_index(t(prior), t(new), table, ps, num_pages=P)
    want = orc.build_index(prior, new, otable, ps, num_pages=P)
    assert_index_equal(index_outputs(idx), want)


def test_reserve_and_index_build_in_a_cuda_graph(cuda):
    """Decode steps as one captured graph: reserve the step's pages, build the
    index, advance the lengths on the device; replayed 40 times with no host
    round trip, then checked against the oracle run step by step."""
    B, W, ps, P = 64, 32, 16, 4096
    rng = np.random.default_rng(5)
    prior0 = rng.integers(1, 200, B).astype(np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    pool, opool = yl.DevicePagePool(P, cuda), orc.PagePool(P)
    table = torch.full((B, W), -1, dtype=torch.int32, device=cuda)
    otable = np.full((B, W), -1, np.int32)
    zeros = np.zeros(B, np.int32)
    pool.reserve(table, t(zeros), t(prior0), ps)
    opool.reserve(otable, zeros, prior0, ps)
    prior, ones = t(prior0), torch.ones(B, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    cap = int(B * W)
    kv_indptr = torch.empty(B + 1, dtype=torch.int32, device=cuda)
    kv_indices = torch.empty(cap, dtype=torch.int32, device=cuda)
    last = torch.empty(B, dtype=torch.int32, device=cuda)
    qo = torch.empty(B + 1, dtype=torch.int32, device=cuda)
    slots = torch.empty(B, dtype=torch.int64, device=cuda)
    out = yl.BatchIndex(kv_indptr, kv_indices, last, qo, slots)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(cuda)
    with torch.cuda.stream(stream):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            pool.reserve(table, prior, ones, ps, error_word=err)
            yl.build_index(prior, ones, table, ps, num_pages=P, out=out, error_word=err)
            prior.add_(ones)
    lens = prior0.copy()
    for _ in range(40):
        g.replay()
        assert opool.reserve(otable, lens, np.ones(B, np.int32), ps) == 0
        want = orc.build_index(lens, np.ones(B, np.int32), otable, ps, num_pages=P)
        lens = lens + 1
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.array_equal(prior.cpu().numpy(), lens)
    assert np.array_equal(table.cpu().numpy(), otable)
    assert np.array_equal(pool.free_list().cpu().numpy(), opool.free_list())
    got = index_outputs(out)
    got["kv_indices"] = got["kv_indices"][:int(want["kv_indptr"][-1])]  # the buffer's defined prefix
    assert_index_equal(got, want)
    del g


def test_cpp_device_pool_matches_host_manager(cuda):
    """DevicePagePool (C++) and the host KVCacheManager, fed the same
    requests, hold the same page table and free-page count."""
    C = yl.load_extension()
    P, R, W, ps = 500, 8, 32, 16
    host = C.KVCacheManager(P, R, W, ps, "cpu")
    rows = [host.AllocateTableSlot() for _ in range(R)]
    dev = C.DevicePagePool(P, "cuda")
    table = torch.full((R, W), -1, dtype=torch.int32, device=cuda)
    rng = np.random.default_rng(11)
    lens = np.zeros(R, np.int64)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    for step in range(20):
        if step % 6 == 5:
            r = int(rng.integers(0, R))
            host.Release(rows[r])
            dev.Release(table, t([rows[r]]), t([lens[r]]), ps)
            rows[r] = host.AllocateTableSlot()
            lens[r] = 0
            continue
        new = np.minimum(rng.integers(0, 50, R), W * ps - lens)
        for i in range(R):
            host.Reserve(rows[i], int(lens[i] + new[i]))
        dev.Reserve(table, t(lens), t(new), ps, t(rows))
        lens += new
    torch.cuda.synchronize()
    assert torch.equal(table.cpu(), host.HostPageTable())
    assert dev.FreeCount() == host.RemainingPageCount()
    with pytest.raises(C.PanicError):
        dev.Reserve(table.to(torch.int64), t(lens), t(lens), ps)
