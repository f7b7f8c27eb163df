"""Pin the CPU oracle before trusting it (no GPU needed).

* index build vs golden vectors produced by the reference's own
  Make2DIndices (tests/golden/index_ps1_*.json, made by make_index_golden.py);
* range expansion vs that helper's own output for multi-range calls
  (tests/golden/make2d_ranges.json, same script);
* index build vs the known answers of the five-request page-size-16 batch;
* C oracle vs the independent pure-Python restatement on seeded random cases;
* store semantics ported from the reference's test/mha_kvcache_test.cpp.
"""
import glob
import json
import os

import numpy as np
import pytest

from oracle import kvpath as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "index_ps1_*.json"))))
def test_index_oracle_matches_reference_make2dindices(path):
    d = json.load(open(path))
    pt = np.array(d["page_table"], np.int32)
    out = orc.build_index(d["prior_len"], d["new_len"], pt, d["page_size"], table_index=d["table_index"])
    assert out["err"] == 0 and out["rc"] == 0
    assert out["kv_indptr"].tolist() == d["kv_indptr"]
    assert out["kv_indices"].tolist() == d["kv_indices"]
    assert out["qo_indptr"].tolist() == d["qo_indptr"]
    assert out["slot_mapping"].tolist() == d["slot_mapping"]
    # page size 1: every non-empty sequence's last page holds one token
    tot = np.array(d["prior_len"]) + np.array(d["new_len"])
    assert out["kv_last_page_len"].tolist() == [1 if t else 0 for t in tot]


def test_make2d_oracle_matches_reference_make2dindices():
    d = json.load(open(os.path.join(GOLDEN, "make2d_ranges.json")))
    assert len(d["calls"]) >= 5
    for call in d["calls"]:
        out, total, bits = orc.make_2d_indices(call["ranges"])
        assert bits == 0 and total == len(call["indices"])
        assert out.tolist() == call["indices"]
        assert orc.py_make_2d_indices(call["ranges"]).tolist() == call["indices"]


def test_make2d_oracle_edge_cases():
    empty, total, bits = orc.make_2d_indices(np.zeros((0, 3), np.int64))
    assert empty.size == 0 and total == 0 and bits == 0
    out, total, bits = orc.make_2d_indices([[10, 2, 5], [0, 4, 4], [100, 0, 2]])
    assert out.tolist() == [12, 13, 14, 100, 101] and bits == 0
    # a negative entry or an inverted range adds nothing
    out, total, bits = orc.make_2d_indices([[-1, 0, 3], [7, 5, 2], [1, 0, 2]])
    assert out.tolist() == [1, 2] and bits == orc.NEGATIVE_LEN
    # row + col_end past INT64_MAX adds nothing
    out, total, bits = orc.make_2d_indices([[2**63 - 2, 0, 5], [3, 0, 1]])
    assert out.tolist() == [3] and bits == orc.INDEX_RANGE
    # capacity: the first `capacity` indices, the total, the bit
    out, total, bits = orc.make_2d_indices([[0, 0, 4], [50, 0, 4]], capacity=6)
    assert out.tolist() == [0, 1, 2, 3, 50, 51] and total == 8 and bits == orc.INDICES_CAP


def test_index_oracle_known_answers_page16():
    # priors 17/33/64/100 with one decode token each, plus a 48-token prefill
    prior = [17, 33, 64, 100, 0]
    fresh = [1, 1, 1, 1, 48]
    W = 8
    pages = (np.arange(5 * W, dtype=np.int32) * 7 + 3).reshape(5, W)
    out = orc.build_index(prior, fresh, pages, 16, num_pages=1024)
    assert out["err"] == 0
    assert out["kv_indptr"].tolist() == [0, 2, 5, 10, 17, 20]
    assert out["kv_last_page_len"].tolist() == [2, 2, 1, 5, 16]
    assert out["qo_indptr"].tolist() == [0, 1, 2, 3, 4, 52]
    s = out["slot_mapping"]
    assert s.shape == (52,)
    assert s[0] == pages[0][1] * 16 + 1          # seq 0: position 17
    assert s[2] == pages[2][4] * 16 + 0          # seq 2: position 64
    assert s[3] == pages[3][6] * 16 + 4          # seq 3: position 100
    assert s[4:].tolist() == [pages[4][t // 16] * 16 + t % 16 for t in range(48)]
    assert out["kv_indices"].tolist() == sum((pages[i][:n].tolist() for i, n in enumerate([2, 3, 5, 7, 3])), [])


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("ps", [1, 16, 64])
def test_index_c_oracle_vs_python(seed, ps):
    rng = np.random.default_rng(seed)
    B = int(rng.integers(1, 40))
    prior = rng.integers(0, 300, B).astype(np.int32)
    fresh = rng.integers(0, 70, B).astype(np.int32)
    prior[rng.random(B) < 0.2] = 0
    fresh[rng.random(B) < 0.2] = 0
    W = int(-(-(prior + fresh).max() // ps)) + 2
    R = B + 5
    pt = rng.permutation(R * W * 2)[: R * W].astype(np.int32).reshape(R, W)
    tix = rng.permutation(R)[:B].astype(np.int32)
    got = orc.build_index(prior, fresh, pt, ps, table_index=tix)
    want = orc.py_build_index(prior, fresh, pt, ps, table_index=tix)
    assert got["err"] == 0
    for name in want:
        assert np.array_equal(got[name], want[name]), name


def test_index_oracle_error_bits():
    pt = np.array([[5, 6], [7, 8]], np.int32)
    # row too short: 3 pages needed, 2 available
    out = orc.build_index([30], [10], pt, 16, max_pages_per_row=2)
    assert out["err"] & orc.ROW_OVERFLOW
    # page id outside the pool
    out = orc.build_index([0], [3], pt, 16, num_pages=6)
    assert out["err"] == 0
    out = orc.build_index([0, 0], [3, 3], pt, 16, num_pages=6)
    assert out["err"] & orc.PAGE_RANGE and out["slot_mapping"][3:].tolist() == [-1, -1, -1]
    # bad table row
    out = orc.build_index([0], [3], pt, 16, table_index=[9])
    assert out["err"] & orc.TABLE_ROW and out["slot_mapping"].tolist() == [-1, -1, -1]
    assert out["kv_indptr"].tolist() == [0, 0]
    # negative lengths count as zero
    out = orc.build_index([-4], [2], pt, 16)
    assert out["err"] & orc.NEGATIVE_LEN and out["slot_mapping"].tolist() == [5 * 16, 5 * 16 + 1]
    # capacities
    out = orc.build_index([0, 0], [20, 20], pt, 16, kv_indices_capacity=3, slot_capacity=30)
    assert out["err"] & orc.INDICES_CAP and out["err"] & orc.SLOTS_CAP


def test_index_oracle_empty_batch():
    out = orc.build_index(np.zeros(0, np.int32), np.zeros(0, np.int32), np.zeros((1, 4), np.int32), 16)
    assert out["kv_indptr"].tolist() == [0] and out["qo_indptr"].tolist() == [0]
    assert out["kv_indices"].size == 0 and out["slot_mapping"].size == 0 and out["err"] == 0


# --- store: behaviours pinned by test/mha_kvcache_test.cpp -----------------
def _rand_rows(rng, shape, dtype=np.float32):
    return rng.standard_normal(shape).astype(dtype)


def test_store_places_rows():  # TestStoreKVStoresCorrectly (mha_kvcache_test.cpp:260-333)
    rng = np.random.default_rng(0)
    H, D, P = 8, 64, 8
    k = _rand_rows(rng, (6, H * D))
    v = _rand_rows(rng, (6, H * D))
    loc = rng.permutation(6).astype(np.int64)
    kc = np.zeros((P, H * D), np.float32)
    vc = np.zeros_like(kc)
    copied, err = orc.store(k, v, kc, vc, loc)
    assert copied == 12 and err == 0
    for i, s in enumerate(loc):
        assert np.array_equal(kc[s], k[i]) and np.array_equal(vc[s], v[i])
    assert not kc[6:].any()


def test_store_second_write_wins():  # TestStoreKVOverwritesSamePage (:338-393)
    rng = np.random.default_rng(1)
    kc = np.zeros((8, 512), np.float32)
    vc = np.zeros_like(kc)
    loc = np.array([1], np.int64)
    k1, v1, k2, v2 = (_rand_rows(rng, (1, 512)) for _ in range(4))
    orc.store(k1, v1, kc, vc, loc)
    orc.store(k2, v2, kc, vc, loc)
    assert np.array_equal(kc[1], k2[0]) and np.array_equal(vc[1], v2[0])


def test_store_empty_is_noop():  # TestStoreKVWithEmptyInput (:398-435)
    kc = np.ones((8, 512), np.float32)
    vc = np.ones_like(kc)
    e = np.zeros((0, 512), np.float32)
    assert orc.store(e, e, kc, vc, np.zeros(0, np.int64)) == (0, 0)
    assert (kc == 1).all() and (vc == 1).all()


def test_store_random_writes_last_writer():  # TestStoreKVMultipleRandomWrites (:473-575), seeded
    rng = np.random.default_rng(3)
    P, E = 128, 512
    kc = np.zeros((P, E), np.float32)
    vc = np.zeros_like(kc)
    last = {}
    for _ in range(500):
        n = int(rng.integers(1, 13))
        loc = rng.permutation(P)[:n].astype(np.int64)
        k = _rand_rows(rng, (n, E))
        v = _rand_rows(rng, (n, E))
        orc.store(k, v, kc, vc, loc)
        for i, s in enumerate(loc):
            last[int(s)] = (k[i].copy(), v[i].copy())
    for s, (kk, vv) in last.items():
        assert np.array_equal(kc[s], kk) and np.array_equal(vc[s], vv)


@pytest.mark.parametrize("threads", [1, 4])
def test_store_c_vs_python_multilayer(threads):
    rng = np.random.default_rng(4)
    L, N, S, E = 3, 37, 200, 96
    k = rng.integers(0, 2**16, (L, N, E), dtype=np.uint16)
    v = rng.integers(0, 2**16, (L, N, E), dtype=np.uint16)
    slots = rng.permutation(S)[:N].astype(np.int32)
    slots[5] = -1  # padding token
    kc = rng.integers(0, 2**16, (L, S, E), dtype=np.uint16)
    vc = kc.copy() ^ 0x5A5A
    kc2, vc2 = kc.copy(), vc.copy()
    copied, err = orc.store(k, v, kc, vc, slots, num_slots=S, threads=threads)
    orc.py_store(k, v, kc2, vc2, slots)
    assert err == 0 and copied == 2 * L * (N - 1)
    assert np.array_equal(kc, kc2) and np.array_equal(vc, vc2)


def test_store_slot_range_error():
    kc = np.zeros((4, 64), np.uint8)
    vc = np.zeros_like(kc)
    k = np.ones((2, 64), np.uint8)
    copied, err = orc.store(k, k, kc, vc, np.array([1, 7], np.int64), num_slots=4)
    assert copied == 2 and err == orc.SLOT_RANGE and kc[1].all() and not kc[[0, 2, 3]].any()


def test_gather_oracle_matches_numpy_take():  # IndexKernel row copy (src/layers/index.cu:61-72)
    rng = np.random.default_rng(5)
    table = rng.integers(0, 1 << 16, size=(300, 96), dtype=np.uint16)
    idx = rng.integers(0, 300, size=1000).astype(np.int32)
    out, err = orc.gather(idx, table)
    assert err == 0 and np.array_equal(out, table[idx])
    out64, _ = orc.gather(idx.astype(np.int64), table)
    assert np.array_equal(out64, out)


def test_gather_oracle_out_of_range_rows_are_zero():
    table = np.arange(40, dtype=np.uint8).reshape(10, 4) + 1
    out, err = orc.gather(np.array([3, -1, 9], np.int64), table)
    assert err == 0 and out[1].sum() == 0 and np.array_equal(out[[0, 2]], table[[3, 9]])
    out, err = orc.gather(np.array([10, 2, -5], np.int64), table)
    assert err == orc.INDEX_RANGE and out[0].sum() == 0 and out[2].sum() == 0 and np.array_equal(out[1], table[2])
    out, err = orc.gather(np.zeros(0, np.int32), table)
    assert out.shape == (0, 4) and err == 0


def test_round_to_matches_torch_conversions():
    import torch

    rng = np.random.default_rng(6)
    x = (rng.standard_normal(100000) * np.exp(rng.uniform(-20, 20, 100000))).astype(np.float32)
    x[:4] = [0.0, -0.0, 1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8]  # ties round to even
    for dtype, tdt in (("bf16", torch.bfloat16), ("fp16", torch.float16)):
        want = torch.from_numpy(x).to(tdt).float().numpy()
        got = orc.round_to(x, dtype)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), dtype


def _qkv_case(N=6, Hq=4, Hk=2, D=64, seed=0, S=32):
    rng = np.random.default_rng(seed)
    r = lambda *s: orc.round_to(rng.standard_normal(s).astype(np.float32), "bf16")
    q, k, v = r(N, Hq, D), r(N, Hk, D), r(N, Hk, D)
    qw, kw = orc.round_to(1 + 0.1 * rng.standard_normal(D).astype(np.float32), "bf16"), r(D)
    pos = rng.integers(0, 100, N)
    ang = pos[:, None] * (1e4 ** (-np.arange(0, D, 2) / D))[None, :]
    cache = np.concatenate([np.cos(np.arange(128)[:, None] * (1e4 ** (-np.arange(0, D, 2) / D))),
                            np.sin(np.arange(128)[:, None] * (1e4 ** (-np.arange(0, D, 2) / D)))], 1).astype(np.float32)
    slots = rng.permutation(S)[:N]
    return q, k, v, qw, kw, pos, cache, slots, ang


@pytest.mark.parametrize("interleaved", [False, True])
def test_qkv_oracle_against_float64_formula(interleaved):
    """The restatement against the textbook formulas in float64 (norm, then
    rotation of pairs by the position's angles)."""
    q, k, v, qw, kw, pos, cache, slots, ang = _qkv_case()
    D = q.shape[-1]
    kc = np.zeros((32, 2, D), np.float32)
    vc = np.zeros_like(kc)
    q_out, err = orc.qkv_norm_rope_store(q, k, v, kc, vc, slots, qw, kw, 1e-6, cache, pos, interleaved)
    assert err == 0

    def ref(x, w):
        x = x.astype(np.float64)
        x = x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * w
        c, s = np.cos(ang)[:, None], np.sin(ang)[:, None]
        a, b = (x[..., 0::2], x[..., 1::2]) if interleaved else (x[..., :D // 2], x[..., D // 2:])
        y = np.empty_like(x)
        if interleaved:
            y[..., 0::2], y[..., 1::2] = a * c - b * s, b * c + a * s
        else:
            y[..., :D // 2], y[..., D // 2:] = a * c - b * s, b * c + a * s
        return y

    np.testing.assert_allclose(q_out, ref(q, qw), atol=3e-2, rtol=3e-2)
    np.testing.assert_allclose(kc[slots], ref(k, kw), atol=3e-2, rtol=3e-2)
    assert np.array_equal(vc[slots], v)


def test_qkv_oracle_error_bits():
    q, k, v, qw, kw, pos, cache, slots, _ = _qkv_case()
    kc = np.zeros((32, 2, 64), np.float32)
    vc = np.zeros_like(kc)
    pos[1], slots[2], slots[3] = 500, -1, 40
    q_out, err = orc.qkv_norm_rope_store(q, k, v, kc, vc, slots, qw, kw, 1e-6, cache, pos)
    assert err == orc.POSITION_RANGE | orc.SLOT_RANGE
    assert np.isnan(q_out[1]).all() and not np.isnan(q_out[[0, 2, 3, 4, 5]]).any()
    written = {int(s) for i, s in enumerate(slots) if i not in (1, 2, 3)}
    assert {int(s) for s in np.nonzero(vc.any(axis=(1, 2)))[0]} == written


def _reference_allocator(P, steps, ps, W):
    """A literal restatement of the reference's AllocateIndices on a Python
    list (cache_manager.h:119-131: return the tail slice, keep the head) plus
    the page-table writes, request by request."""
    free = list(range(P))
    table = [[-1] * W for _ in range(len(steps[0][1]))]
    for op, a, b in steps:
        if op == "reserve":
            for i, (prior, new) in enumerate(zip(a, b)):
                held, need = -(-prior // ps), -(-(prior + new) // ps)
                size = need - held
                if size:
                    got, free = free[len(free) - size:], free[:len(free) - size]
                    table[i][held:need] = got
        else:
            for row, toks in zip(a, b):
                c = -(-toks // ps)
                free += table[row][:c]
                table[row][:c] = [-1] * c
    return free, table


@pytest.mark.parametrize("ps", [1, 16])
def test_page_pool_oracle_matches_list_restatement(ps):
    rng = np.random.default_rng(ps)
    B, W, P = 12, 64, 800
    lens = np.zeros(B, np.int64)
    steps = []
    for _ in range(30):
        if rng.random() < 0.3:
            rows = rng.choice(B, size=3, replace=False)
            steps.append(("release", rows.tolist(), lens[rows].tolist()))
            lens[rows] = 0
        else:
            new = rng.integers(0, 3 * ps, B)
            new = np.minimum(new, W * ps - lens)
            steps.append(("reserve", lens.tolist(), new.tolist()))
            lens += new
    pool = orc.PagePool(P)
    table = np.full((B, W), -1, np.int32)
    for op, a, b in steps:
        err = pool.reserve(table, a, b, ps) if op == "reserve" else pool.release(table, a, b, ps)
        assert err == 0
    free, want = _reference_allocator(P, [(op, a, b) if op == "release" else (op, a, b) for op, a, b in steps], ps, W)
    assert pool.free_list().tolist() == free
    assert table.tolist() == want


def test_page_pool_oracle_is_all_or_nothing():
    pool = orc.PagePool(10)
    table = np.full((3, 8), -1, np.int32)
    assert pool.reserve(table, [0, 0], [16, 30], 4) == orc.POOL_EMPTY  # 4 + 8 pages > 10 free
    assert pool.reserve(table, [0, 0], [16, 33], 4) == 0x4  # second row would need 9 > 8 pages
    assert pool.reserve(table, [0, -1], [4, 4], 4) == 0x20
    assert pool.reserve(table, [0, 0], [4, 4], 4, table_index=[0, 3]) == 0x80
    assert (table == -1).all() and pool.count[0] == 10
    assert pool.reserve(table, [0, 0], [8, 4], 4) == 0
    # request 0 takes the tail [8, 9], request 1 the next tail [7]
    assert table[0, :2].tolist() == [8, 9] and table[1, :1].tolist() == [7] and pool.count[0] == 7
    before = table.copy()
    assert pool.reserve(table, [0, 0], [4, 4], 4, table_index=[2, 2]) == orc.DUPLICATE_ROW  # row 2 twice
    assert pool.release(table, [0, 0], [8, 8], 4) == orc.DUPLICATE_ROW  # row 0's pages would enter twice
    assert np.array_equal(table, before) and pool.count[0] == 7
    full = orc.PagePool(10, free_pages=np.arange(9, dtype=np.int32))
    assert full.release(table, [0], [8], 4) == orc.POOL_OVERFLOW and full.count[0] == 9  # 9 + 2 > 10
    assert pool.release(table, [1, 0], [4, 8], 4) == 0 and pool.free_list().tolist() == list(range(7)) + [7, 8, 9]
    assert pool.reserve(table, [0, 0], [8, 4], 4) == 0 and pool.count[0] == 7  # back to the state above
    assert pool.release(table, [0], [8], 4) == 0 and pool.free_list().tolist() == list(range(7)) + [8, 9]
    assert pool.release(table, [1], [4], 4) == 0 and pool.free_list().tolist() == list(range(7)) + [8, 9, 7]
    bad = np.array([[5, 11, -1, -1, -1, -1, -1, -1]] * 3, np.int32)
    assert pool.release(bad, [0], [8], 4) == 0x2 and pool.count[0] == 10  # page id 11 outside the pool


def test_host_kvcache_manager_matches_page_pool_oracle():
    """The C++ front end's host KVCacheManager (Reserve / Release, one request
    at a time) and the oracle give the same page table and free list."""
    import torch

    import yllang_b200 as yl

    C = yl.load_extension()
    P, R, W, ps = 300, 6, 32, 16
    m = C.KVCacheManager(P, R, W, ps, "cpu")
    rows = [m.AllocateTableSlot() for _ in range(R)]
    pool = orc.PagePool(P)
    table = np.full((R, W), -1, np.int32)
    rng = np.random.default_rng(9)
    lens = np.zeros(R, np.int64)
    for step in range(25):
        if step % 7 == 6:
            r = int(rng.integers(0, R))
            m.Release(rows[r])
            assert pool.release(table, [rows[r]], [int(lens[r])], ps) == 0
            rows[r] = m.AllocateTableSlot()
            lens[r] = 0
            continue
        new = np.minimum(rng.integers(0, 40, R), W * ps - lens)
        for i in range(R):
            m.Reserve(rows[i], int(lens[i] + new[i]))
        assert pool.reserve(table, lens, new, ps, table_index=np.array(rows)) == 0
        lens += new
    assert np.array_equal(m.HostPageTable().numpy(), table)
    assert m.RemainingPageCount() == int(pool.count[0])


@pytest.mark.parametrize("which", ["cpu_ref", "decode", "mixed_ps1", "mixed_ps64"])
def test_torch_restatement_matches_c_oracle(which):
    """The libtorch CPU restatement the CPU baseline times gives the C oracle's
    index arrays and pool bytes."""
    import torch
    from yllang_b200 import workloads
    b = {"cpu_ref": lambda: workloads.cpu_ref(),
         "decode": lambda: workloads.llama3_decode(80000, layers=2),
         "mixed_ps1": lambda: workloads.mixed(20000, page_size=1, head_dim=64, layers=2),
         "mixed_ps64": lambda: workloads.mixed(6000, page_size=64, head_dim=256, layers=2)}[which]()
    want = orc.build_index(b.prior_len, b.new_len, b.page_table, b.page_size)
    got = orc.torch_build_index(torch.from_numpy(b.prior_len), torch.from_numpy(b.new_len),
                                torch.from_numpy(b.page_table), b.page_size)
    for name in got:
        assert np.array_equal(got[name].numpy(), want[name]), name
    S, E = b.num_pages * b.page_size, 64
    rng = np.random.default_rng(5)
    k = rng.integers(-2**15, 2**15, (b.layers, b.tokens, E), dtype=np.int16)
    v = rng.integers(-2**15, 2**15, (b.layers, b.tokens, E), dtype=np.int16)
    pools = rng.integers(-2**15, 2**15, (2, b.layers, S, E), dtype=np.int16)
    want_pools = pools.copy()
    orc.store(k, v, want_pools[0], want_pools[1], want["slot_mapping"])
    tp = torch.from_numpy(pools)
    orc.torch_store(torch.from_numpy(k), torch.from_numpy(v), tp[0], tp[1], got["slot_mapping"])
    assert np.array_equal(tp.numpy(), want_pools)
