"""Batch index build on the GPU vs the CPU oracle and the reference's own
golden vectors, through the C ABI (bit-exact, integer work)."""
import glob
import json
import os

import numpy as np
import pytest
import torch

import yllang_b200 as yl
from _kvutil import assert_index_equal, index_outputs
from oracle import kvpath as orc
from yllang_b200 import workloads

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _run(dev, prior, new, table, ps, table_index=None, num_pages=0, slot_dtype=torch.int64, kv_cap=None,
         slot_cap=None, max_pages_per_row=None):
    """GPU build and oracle build of the same batch; returns (got, want, err)."""
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)
    table = np.ascontiguousarray(table, np.int32)
    tab = t(table)
    if max_pages_per_row is not None:
        tab = tab[:, :max_pages_per_row]
    want = orc.build_index(prior, new, table if max_pages_per_row is None else table[:, :max_pages_per_row], ps,
                           table_index=table_index, num_pages=num_pages,
                           slot_dtype=np.int64 if slot_dtype == torch.int64 else np.int32,
                           kv_indices_capacity=kv_cap, slot_capacity=slot_cap)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    idx = yl.build_index(t(prior), t(new), tab, ps, table_index=None if table_index is None else t(table_index),
                         num_pages=num_pages, slot_dtype=slot_dtype, error_word=err,
                         kv_indices_capacity=want["kv_indices"].size, slot_capacity=want["slot_mapping"].size)
    torch.cuda.synchronize()
    return index_outputs(idx), want, int(err.item())


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "index_ps1_*.json"))))
def test_index_matches_reference_golden(cuda, path):
    d = json.load(open(path))
    got, want, err = _run(cuda, d["prior_len"], d["new_len"], d["page_table"], 1, table_index=d["table_index"])
    assert err == 0
    assert got["kv_indptr"].tolist() == d["kv_indptr"]
    assert got["kv_indices"].tolist() == d["kv_indices"]
    assert got["qo_indptr"].tolist() == d["qo_indptr"]
    assert got["slot_mapping"].tolist() == d["slot_mapping"]


def test_index_known_answers_page16(cuda):
    pages = (np.arange(40, dtype=np.int32) * 7 + 3).reshape(5, 8)
    got, want, err = _run(cuda, [17, 33, 64, 100, 0], [1, 1, 1, 1, 48], pages, 16, num_pages=1024)
    assert err == 0
    assert got["kv_indptr"].tolist() == [0, 2, 5, 10, 17, 20]
    assert got["kv_last_page_len"].tolist() == [2, 2, 1, 5, 16]
    assert got["qo_indptr"].tolist() == [0, 1, 2, 3, 4, 52]
    assert_index_equal(got, want)


@pytest.mark.parametrize("seed", range(8))
@pytest.mark.parametrize("ps", [1, 16, 64])
@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64])
def test_index_random_batches(cuda, seed, ps, slot_dtype):
    rng = np.random.default_rng(seed * 31 + ps)
    B = int(rng.integers(1, 3000))
    prior = rng.integers(0, 5000, B).astype(np.int32)
    new = rng.integers(0, 300, B).astype(np.int32)
    prior[rng.random(B) < 0.1] = 0
    new[rng.random(B) < 0.1] = 0
    W = int(-(-(prior.astype(np.int64) + new).max() // ps)) + 1
    R = B + 7
    table = rng.integers(0, 1 << 20, (R, W)).astype(np.int32)
    tix = rng.permutation(R)[:B].astype(np.int32) if seed % 2 else None
    if tix is None:
        table = table[:B]
    got, want, err = _run(cuda, prior, new, table, ps, table_index=tix, slot_dtype=slot_dtype)
    assert err == 0
    assert_index_equal(got, want)


@pytest.mark.parametrize("name", ["cpu_ref", "llama3_decode", "ragged_prefill", "qwen72b_decode", "mixed"])
def test_index_workloads(cuda, name):
    if name == "cpu_ref":
        batches = [workloads.cpu_ref()]
    elif name == "llama3_decode":
        batches = [workloads.llama3_decode(num_pages=71525)]
    elif name == "ragged_prefill":
        batches = [workloads.ragged_prefill(num_pages=71525)]
    elif name == "qwen72b_decode":
        batches = [workloads.qwen72b_decode(num_pages=28610, tp=1), workloads.qwen72b_decode(num_pages=228881, tp=8)]
    else:
        batches = [workloads.mixed(num_pages=50000, page_size=ps, head_dim=hd) for ps in (1, 16, 64)
                   for hd in (64, 128, 256)]
    for b in batches:
        got, want, err = _run(cuda, b.prior_len, b.new_len, b.page_table, b.page_size, num_pages=b.num_pages)
        assert err == 0, b.name
        assert_index_equal(got, want)
        assert got["kv_indptr"][-1] == b.total_pages and got["qo_indptr"][-1] == b.tokens


def test_index_large_batch_two_launch_form(cuda):
    # batches above the shared-memory limit (16384 sequences) scan into the outputs first
    rng = np.random.default_rng(5)
    B = 20000
    prior = rng.integers(0, 400, B).astype(np.int32)
    new = rng.integers(0, 3, B).astype(np.int32)
    W = int(-(-(prior + new).max() // 16)) + 1
    table = rng.integers(0, 1 << 22, (B, W)).astype(np.int32)
    got, want, err = _run(cuda, prior, new, table, 16)
    assert err == 0
    assert_index_equal(got, want)


@pytest.mark.parametrize("B,tix", [(2048, False), (3000, True), (20000, False)])
def test_index_big_batch_errors_and_capacity(cuda, B, tix):
    """Decode-shaped big batches (the warp-per-sequence page copy; 20,000 in
    the two-launch form) with page ids outside the pool and a kv_indices
    capacity below the batch's pages: same outputs and error bits as the
    oracle."""
    rng = np.random.default_rng(B)
    prior = rng.integers(100, 4000, B).astype(np.int32)
    new = np.ones(B, np.int32)
    ps, P = 16, 1 << 20
    W = int(-(-(prior.astype(np.int64) + new).max() // ps)) + 1
    R = B + 11 if tix else B
    table = rng.integers(0, P, (R, W)).astype(np.int32)
    rows = rng.permutation(R)[:B].astype(np.int32) if tix else None
    first = rows[:5] if tix else np.arange(5)
    table[first, rng.integers(0, 4, 5)] = P + 7  # outside the pool, in pages the first sequences hold
    total = int(((prior.astype(np.int64) + new + ps - 1) // ps).sum())
    got, want, err = _run(cuda, prior, new, table, ps, table_index=rows, num_pages=P, kv_cap=total - 1000)
    assert want["err"] & orc.INDICES_CAP and err == want["err"]
    assert_index_equal(got, want)


def test_index_empty_and_zero_length(cuda):
    got, want, err = _run(cuda, np.zeros(0, np.int32), np.zeros(0, np.int32), np.zeros((1, 4), np.int32), 16)
    assert err == 0 and got["kv_indptr"].tolist() == [0] and got["qo_indptr"].tolist() == [0]
    got, want, err = _run(cuda, [0, 5, 0, 16], [0, 0, 3, 0], np.arange(16, dtype=np.int32).reshape(4, 4), 16)
    assert err == 0
    assert_index_equal(got, want)
    assert got["kv_last_page_len"].tolist() == [0, 5, 3, 16]


def test_index_error_bits_match_oracle(cuda):
    table = np.array([[5, 6], [7, 8]], np.int32)
    cases = [
        dict(prior=[30], new=[10], max_pages_per_row=2, bit=orc.ROW_OVERFLOW),
        dict(prior=[0, 0], new=[3, 3], num_pages=6, bit=orc.PAGE_RANGE),
        dict(prior=[0], new=[3], table_index=[9], bit=orc.TABLE_ROW),
        dict(prior=[-4], new=[2], bit=orc.NEGATIVE_LEN),
        dict(prior=[0, 0], new=[20, 20], kv_cap=3, slot_cap=30, bit=orc.INDICES_CAP | orc.SLOTS_CAP),
    ]
    for c in cases:
        prior = np.array(c["prior"], np.int32)
        new = np.array(c["new"], np.int32)
        tab = table if "table_index" in c else table[: len(prior)]
        mp = c.get("max_pages_per_row")
        want = orc.build_index(prior, new, tab if mp is None else tab[:, :mp], 16, table_index=c.get("table_index"),
                               num_pages=c.get("num_pages", 0), kv_indices_capacity=c.get("kv_cap"),
                               slot_capacity=c.get("slot_cap"))
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        tix = c.get("table_index")
        idx = yl.build_index(t(prior), t(new), t(tab)[:, :mp] if mp else t(tab), 16,
                             table_index=None if tix is None else t(tix), num_pages=c.get("num_pages", 0),
                             error_word=err, kv_indices_capacity=want["kv_indices"].size,
                             slot_capacity=want["slot_mapping"].size)
        torch.cuda.synchronize()
        assert int(err.item()) == want["err"] and want["err"] & c["bit"], c
        assert_index_equal(index_outputs(idx), want)


def test_index_then_store_step(cuda):
    """One step of the path: index build feeds its slot mapping to the store."""
    b = workloads.cpu_ref()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    idx = yl.build_index(t(b.prior_len), t(b.new_len), t(b.page_table), b.page_size, num_pages=b.num_pages,
                         kv_indices_capacity=b.total_pages, slot_capacity=b.tokens)
    E = b.kv_heads * b.head_dim
    torch.manual_seed(0)
    k = torch.randn(b.tokens, E).to(torch.bfloat16).to(cuda)
    v = torch.randn(b.tokens, E).to(torch.bfloat16).to(cuda)
    S = b.num_pages * b.page_size
    kc = torch.zeros(S, E, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    yl.store_kv_cache(k, v, kc, vc, idx.slot_mapping)
    torch.cuda.synchronize()
    want = orc.build_index(b.prior_len, b.new_len, b.page_table, b.page_size)["slot_mapping"]
    s = torch.from_numpy(want).to(cuda)
    assert torch.equal(kc[s].view(torch.int16), k.view(torch.int16))
    assert torch.equal(vc[s].view(torch.int16), v.view(torch.int16))
