"""Range expansion (yl_make_2d_indices, the reference's Make2DIndices,
src/include/batch/batch_manager.h:30-51) on the GPU, bit-exact against the
helper's own output (tests/golden/make2d_ranges.json) and the oracle: ranges
across several 512-range scan chunks, empty and invalid ranges, a short
output buffer, one long range spread over the whole grid, the C++ front end
with the reference's float range tensors, and NextBatch's use of the indices
on a page table (batch_manager.h:104-112)."""
import glob
import json
import os

import numpy as np
import pytest
import torch

import yllang_b200 as yl
from oracle import kvpath as orc

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _ranges(rng, n, max_row=10**6, max_col=400, empty_every=7):
    row = rng.integers(0, max_row, n)
    lo = rng.integers(0, max_col, n)
    hi = lo + rng.integers(0, max_col, n)
    hi[::empty_every] = lo[::empty_every]
    return np.stack([row, lo, hi], axis=1).astype(np.int64)


def test_make2d_matches_reference_helper_output(cuda):
    d = json.load(open(os.path.join(GOLDEN, "make2d_ranges.json")))
    C = yl.load_extension()
    table = torch.zeros(8, 8, device=cuda)
    for call in d["calls"]:
        r = torch.tensor(call["ranges"], dtype=torch.int64, device=cuda)
        got = yl.make_2d_indices(r)
        # the C++ front end, fed range tensors as NextBatch builds them (torch::empty(3), float)
        cpp = C.Make2DIndices(table, [torch.tensor(x, dtype=torch.float32) for x in call["ranges"]])
        torch.cuda.synchronize()
        assert got.cpu().tolist() == call["indices"]
        assert cpp.dtype == torch.int64 and cpp.device == table.device
        assert cpp.cpu().tolist() == call["indices"]


@pytest.mark.parametrize("n", [1, 31, 511, 512, 513, 1500, 5000])
def test_make2d_random_ranges_vs_oracle(cuda, n):
    rng = np.random.default_rng(n)
    r = _ranges(rng, n)
    want, total, bits = orc.make_2d_indices(r)
    assert bits == 0
    dr = torch.from_numpy(r).to(cuda)
    got = yl.make_2d_indices(dr)
    count = torch.full((1,), -1, dtype=torch.int64, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.full((total + 64,), -5, dtype=torch.int64, device=cuda)
    yl.make_2d_indices(dr, out=out, count=count, error_word=err)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), want)
    assert np.array_equal(out[:total].cpu().numpy(), want)
    assert bool((out[total:] == -5).all())
    assert int(count.item()) == total and int(err.item()) == 0


def test_make2d_short_output_and_invalid_ranges(cuda):
    rng = np.random.default_rng(3)
    r = _ranges(rng, 900)
    r[10] = [-4, 0, 5]              # negative row
    r[600] = [7, 9, 3]              # col_end < col_start
    r[700] = [2**63 - 10, 0, 50]    # row + col_end past INT64_MAX
    dr = torch.from_numpy(r).to(cuda)
    for cap in (0, 1, 1000, 60000):
        want, total, bits = orc.make_2d_indices(r, capacity=cap)
        buf = torch.full((cap + 32,), -5, dtype=torch.int64, device=cuda)
        count = torch.zeros(1, dtype=torch.int64, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        yl.make_2d_indices(dr, out=buf[:cap], count=count, error_word=err)
        torch.cuda.synchronize()
        m = min(total, cap)
        assert np.array_equal(buf[:m].cpu().numpy(), want)
        assert bool((buf[m:] == -5).all())
        assert int(count.item()) == total and int(err.item()) == bits
        assert bits & orc.NEGATIVE_LEN and bits & orc.INDEX_RANGE
        assert bool(bits & orc.INDICES_CAP) == (total > cap)
    with pytest.raises(yl.PanicError):
        yl.make_2d_indices(dr)  # without an output buffer, invalid ranges are refused on the host


def test_make2d_empty_and_long_ranges(cuda):
    count = torch.full((1,), -1, dtype=torch.int64, device=cuda)
    out = torch.empty(4, dtype=torch.int64, device=cuda)
    yl.make_2d_indices(torch.zeros(0, 3, dtype=torch.int64, device=cuda), out=out, count=count)
    torch.cuda.synchronize()
    assert int(count.item()) == 0
    assert yl.make_2d_indices(torch.tensor([[5, 3, 3], [9, 0, 0]], dtype=torch.int64, device=cuda)).numel() == 0
    # one range of 3 M indices between two short ones: every block of the grid writes
    r = np.array([[11, 2, 9], [1 << 40, 5, 5 + 3_000_000], [0, 0, 3]], np.int64)
    want, total, _ = orc.make_2d_indices(r)
    got = yl.make_2d_indices(torch.from_numpy(r).to(cuda))
    torch.cuda.synchronize()
    assert got.numel() == total and np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "index_ps1_*.json"))))
def test_make2d_drives_next_batch_page_lookup(cuda, path):
    """NextBatch's use (batch_manager.h:97-112): load ranges {row * W, 0,
    device_len} and write ranges {row * W, cached_len, device_len} over the
    page table; the flat table entries they pick are the kv_indices and slot
    mapping the reference's helper gives (page size 1)."""
    d = json.load(open(path))
    pt = torch.tensor(d["page_table"], dtype=torch.int32, device=cuda)
    W = pt.shape[1]
    rows = np.array(d["table_index"], np.int64)
    prior, fresh = np.array(d["prior_len"], np.int64), np.array(d["new_len"], np.int64)
    load = np.stack([rows * W, np.zeros_like(rows), prior + fresh], axis=1)
    write = np.stack([rows * W, prior, prior + fresh], axis=1)
    flat = pt.view(-1)
    kv_indices = flat[yl.make_2d_indices(torch.from_numpy(load).to(cuda))]
    slots = flat[yl.make_2d_indices(torch.from_numpy(write).to(cuda))]
    torch.cuda.synchronize()
    assert kv_indices.cpu().tolist() == d["kv_indices"]
    assert slots.cpu().tolist() == d["slot_mapping"]


def test_cpp_make2d_range_tensors_and_checks(cuda):
    """yllang::Make2DIndices takes range tensors of any dtype on the host or
    the device (the first three entries of each), and refuses what the
    reference's size_t arithmetic would wrap."""
    C = yl.load_extension()
    table = torch.zeros(4, 4, device=cuda)
    want = [10, 11, 12, 40, 41]
    for make in (lambda x: torch.tensor(x, dtype=torch.int64, device=cuda),
                 lambda x: torch.tensor(x, dtype=torch.int32),
                 lambda x: torch.tensor(x + [99], dtype=torch.float64)):
        got = C.Make2DIndices(table, [make([10, 0, 3]), make([5, 2, 2]), make([40, 0, 2])])
        torch.cuda.synchronize()
        assert got.cpu().tolist() == want
    assert C.Make2DIndices(table, []).numel() == 0
    for bad in ([-1, 0, 2], [0, 3, 1], [0, -2, 1]):
        with pytest.raises(C.PanicError):
            C.Make2DIndices(table, [torch.tensor(bad)])
    with pytest.raises(C.PanicError, match="three entries"):
        C.Make2DIndices(table, [torch.tensor([1, 2])])
    with pytest.raises(C.PanicError, match="different devices"):
        C.Make2DIndices(table, [torch.tensor([0, 0, 1]), torch.tensor([0, 0, 1], device=cuda)])
