"""Generate index-build golden vectors from the reference's own host code.

Run in a tree where the reference harness oracle/_ref/libref_index.so has
been built (``make -C oracle ref``); writes tests/golden/index_ps1_*.json and
tests/golden/make2d_ranges.json (the helper's own output for multi-range
calls).

The reference's only index code is Make2DIndices
(src/include/batch/batch_manager.h:30-51), which NextBatch calls with one
{table_index, cached_len, device_len} range per request
(batch_manager.h:97-107) over a page table whose entries are slots
(page_size 1, src/include/kvcache/mha_kvcache.h:144).  For each request:

    load indices  = Make2DIndices(table, {row * W, 0, device_len})
    write indices = Make2DIndices(table, {row * W, cached_len, device_len})
    kv_indices    = page_table.flat[load indices]     (the pages attention reads)
    slot_mapping  = page_table.flat[write indices]    (the slots the store writes)

The row entry is passed as row * W because Make2DIndices adds the row
number without the row stride (batch_manager.h:43-44); everything else is
the helper's own output.  kv_indptr / qo_indptr are the running sums of the
per-request output lengths the helper returns.
"""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libref_index.so")


def _ref():
    L = ctypes.CDLL(REF_LIB)
    f = L.ref_make2d_indices
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.POINTER(ctypes.c_int64)]
    return f


def make2d(f, rows, cols, ranges):
    ranges = np.ascontiguousarray(ranges, np.int64).reshape(-1, 3)
    cap = int(max(1, (ranges[:, 2] - ranges[:, 1]).clip(min=0).sum()))
    out = np.zeros(cap, np.float32)
    n = ctypes.c_int64(0)
    rc = f(rows, cols, ranges.ctypes.data, ranges.shape[0], out.ctypes.data, cap, ctypes.byref(n))
    assert rc == 0, rc
    return out[: n.value].astype(np.int64)


def case(f, name, page_table, table_index, cached, device):
    R, W = page_table.shape
    flat = page_table.reshape(-1)
    kv_indices, slots, kv_indptr, qo_indptr = [], [], [0], [0]
    for row, c, d in zip(table_index, cached, device):
        load = make2d(f, R, W, [[row * W, 0, d]])
        write = make2d(f, R, W, [[row * W, c, d]])
        kv_indices += flat[load].tolist()
        slots += flat[write].tolist()
        kv_indptr.append(kv_indptr[-1] + len(load))
        qo_indptr.append(qo_indptr[-1] + len(write))
    doc = {
        "name": name,
        "source": "reference Make2DIndices (src/include/batch/batch_manager.h:30-51) via oracle/_ref/libref_index.so",
        "page_size": 1,
        "page_table": page_table.tolist(),
        "table_index": [int(x) for x in table_index],
        "prior_len": [int(x) for x in cached],
        "new_len": [int(d - c) for c, d in zip(cached, device)],
        "kv_indptr": kv_indptr,
        "kv_indices": kv_indices,
        "qo_indptr": qo_indptr,
        "slot_mapping": slots,
    }
    with open(os.path.join(HERE, f"index_ps1_{name}.json"), "w") as fh:
        json.dump(doc, fh, separators=(",", ":"))
    return doc


def make2d_cases(f):
    """Make2DIndices calls as NextBatch makes them (one {row, cached, device}
    range per request, all requests in one call), with the row entries as
    given (the helper adds them without a row stride) and as row * W."""
    rng = np.random.default_rng(11)
    calls = []
    for n, W, scale in ((1, 64, 1), (5, 128, 1), (5, 128, 0), (37, 512, 1), (700, 96, 1)):
        rows = rng.permutation(max(n, 8))[:n]
        cached = rng.integers(0, W // 2, n)
        device = cached + rng.integers(0, W // 2, n)
        if n > 3:
            device[1] = cached[1]          # an empty range
            cached[2], device[2] = 0, 0    # another
        ranges = np.stack([rows * (W if scale else 1), cached, device], axis=1).astype(np.int64)
        out = make2d(f, max(n, 8), W, ranges)
        calls.append({"ranges": ranges.tolist(), "indices": out.tolist()})
    doc = {"source": "reference Make2DIndices (src/include/batch/batch_manager.h:30-51) via oracle/_ref/libref_index.so",
           "calls": calls}
    with open(os.path.join(HERE, "make2d_ranges.json"), "w") as fh:
        json.dump(doc, fh, separators=(",", ":"))


def main():
    f = _ref()
    # The five requests of the 1-layer CPU config at page size 1: cached
    # 17/33/64/100 plus one decode token each, and a 48-token prefill.
    rng = np.random.default_rng(2)
    W = 128
    table = rng.permutation(1024 * 16)[: 8 * W].astype(np.int32).reshape(8, W)
    case(f, "five_requests", table, [0, 1, 2, 3, 4], [17, 33, 64, 100, 0], [18, 34, 65, 101, 48])
    # Ragged mix with permuted page-table rows, zero-token and empty requests.
    rng = np.random.default_rng(7)
    W = 256
    R = 64
    table = rng.permutation(R * W * 4)[: R * W].astype(np.int32).reshape(R, W)
    rows = rng.permutation(R)[:32]
    cached = rng.integers(0, 200, 32)
    extend = rng.integers(0, 41, 32)
    extend[3] = 0
    cached[5], extend[5] = 0, 0
    device = cached + extend
    case(f, "ragged_permuted_rows", table, rows, cached, device)
    make2d_cases(f)


if __name__ == "__main__":
    main()
