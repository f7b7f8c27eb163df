"""Python face of the CPU oracle for the paged KV store and batch index build.

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
to compare the GPU results against, and by bench.py's CPU-baseline leg.  The
product package (``yllang_b200``) never imports it.

Two restatements of the reference's algorithm live here:

* the C oracle (``kvpath_oracle.c``, built into ``liboracle_kvpath.so``), the
  one the tests and the CPU baseline use;
* pure-Python loops (``py_store`` / ``py_build_index``) for small cases, a
  second, independent statement used to cross-check the C one.

The store follows StoreKVCacheKernel (src/kvcache/store_kv_cache.cu:60-72) as
driven by MHAKVCache::StoreKV (src/include/kvcache/mha_kvcache.h:76-86); the
index build follows the request ranges of BatchManager::NextBatch
(src/include/batch/batch_manager.h:97-112) generalised to page_size >= 1.
Argument meanings and error bits are those of include/yl_kvpath.h.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_kvpath.so")
_lib = None

SLOT_RANGE = 0x1
PAGE_RANGE = 0x2
ROW_OVERFLOW = 0x4
INDICES_CAP = 0x8
SLOTS_CAP = 0x10
NEGATIVE_LEN = 0x20
INDPTR_OVERFLOW = 0x40
TABLE_ROW = 0x80
INDEX_RANGE = 0x400
POSITION_RANGE = 0x800
POOL_EMPTY = 0x1000
POOL_OVERFLOW = 0x2000
DUPLICATE_ROW = 0x4000

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_vp = ctypes.c_void_p


def build(with_reference: bool = False) -> None:
    """Compile the oracle (and, if asked and present, the reference harnesses)."""
    target = ["all", "ref"] if with_reference else ["all"]
    env = dict(os.environ)
    # The C oracle is plain C11 + pthreads: any gcc works.
    env.setdefault("CC", "gcc")
    subprocess.run(["make", "-s", "-C", _HERE, *target], check=True, env=env)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "kvpath_oracle.c")
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(src) > os.path.getmtime(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_kv_store.restype = _i64
        L.oracle_kv_store.argtypes = [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, _i64, _i64, _i64, _i64, _i64, _i32,
                                      _i64, _i64, _i64, _i64, _vp, ctypes.c_int]
        L.oracle_build_index.restype = ctypes.c_int
        L.oracle_build_index.argtypes = [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i64, _vp, _vp, _vp, _vp,
                                         _vp, ctypes.c_int, _i64, _i64, _vp]
        L.oracle_max_threads.restype = ctypes.c_int
        L.oracle_reserve_pages.restype = ctypes.c_uint32
        L.oracle_reserve_pages.argtypes = [_vp, _vp, _i64, _vp, _i64, ctypes.c_int32, ctypes.c_int32, _vp, _vp, _vp,
                                           ctypes.c_int32, ctypes.c_int32]
        L.oracle_release_pages.restype = ctypes.c_uint32
        L.oracle_release_pages.argtypes = [_vp, _vp, _i64, _vp, _i64, ctypes.c_int32, ctypes.c_int32, _vp, _vp,
                                           ctypes.c_int32, ctypes.c_int32]
        L.oracle_gather_rows.restype = _i64
        L.oracle_gather_rows.argtypes = [_vp, _vp, _vp, ctypes.c_int, _i64, _i64, _i64, _i64, _i64, _vp]
        L.oracle_make_2d_indices.restype = ctypes.c_uint32
        L.oracle_make_2d_indices.argtypes = [_vp, _i64, _vp, _i64, _vp]
        _lib = L
    return _lib


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def _ptr(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data


def _as3(a: np.ndarray) -> np.ndarray:
    return a[None] if a.ndim == 2 else a


def store(k: np.ndarray, v: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, slots: np.ndarray,
          num_slots: int = 0, threads: int = 1) -> tuple[int, int]:
    """Scatter K/V rows into the caches in place; returns (rows copied, error bits).

    k, v: [N, E] or [L, N, E]; k_cache, v_cache: [S, E] or [L, S, E] (the
    pool's per-layer [pages * page_size, H * D] views); any dtype, rows must be
    contiguous in their last axis; slots int32 or int64 [N].
    """
    k3, v3, kc3, vc3 = _as3(k), _as3(v), _as3(k_cache), _as3(v_cache)
    L, N, E = k3.shape
    if N == 0:  # MHAKVCache::StoreKV returns early (mha_kvcache.h:77-79)
        return 0, 0
    item = k3.itemsize
    for a in (k3, v3, kc3, vc3):
        assert a.strides[2] == item and a.shape[2] == E and a.itemsize == item
    assert kc3.strides == vc3.strides and kc3.shape == vc3.shape and v3.shape == k3.shape
    assert slots.dtype in (np.int32, np.int64) and slots.shape == (N,) and slots.flags.c_contiguous
    err = ctypes.c_uint32(0)
    copied = lib().oracle_kv_store(
        _ptr(k3), _ptr(v3), _ptr(kc3), _ptr(vc3), _ptr(slots), int(slots.dtype == np.int64), N, E * item,
        k3.strides[1], v3.strides[1], kc3.strides[1], L, k3.strides[0], v3.strides[0], kc3.strides[0],
        int(num_slots), ctypes.addressof(err), int(threads))
    return int(copied), int(err.value)


def build_index(prior_len, new_len, page_table: np.ndarray, page_size: int, table_index=None, num_pages: int = 0,
                max_pages_per_row: int | None = None, slot_dtype=np.int64, kv_indices_capacity: int | None = None,
                slot_capacity: int | None = None) -> dict:
    """Index build on the host.  Returns the five arrays plus 'err' and 'rc'."""
    prior = np.ascontiguousarray(prior_len, dtype=np.int32)
    fresh = np.ascontiguousarray(new_len, dtype=np.int32)
    B = prior.shape[0]
    pt = np.ascontiguousarray(page_table, dtype=np.int32)
    if pt.ndim == 1:
        pt = pt[None]
    tix = None if table_index is None else np.ascontiguousarray(table_index, dtype=np.int32)
    mppr = pt.shape[1] if max_pages_per_row is None else max_pages_per_row
    tot = prior.astype(np.int64).clip(min=0) + fresh.astype(np.int64).clip(min=0)
    if kv_indices_capacity is None:
        kv_indices_capacity = int(np.minimum((tot + page_size - 1) // page_size, mppr).sum()) if B else 0
    if slot_capacity is None:
        slot_capacity = int(fresh.astype(np.int64).clip(min=0).sum())
    out = {
        "kv_indptr": np.zeros(B + 1, np.int32),
        "kv_indices": np.zeros(max(kv_indices_capacity, 1), np.int32),
        "kv_last_page_len": np.zeros(max(B, 1), np.int32),
        "qo_indptr": np.zeros(B + 1, np.int32),
        "slot_mapping": np.zeros(max(slot_capacity, 1), slot_dtype),
    }
    err = ctypes.c_uint32(0)
    rc = lib().oracle_build_index(
        _ptr(prior), _ptr(fresh), _ptr(pt), _ptr(tix), pt.strides[0] // 4, pt.shape[0], mppr, page_size, B,
        int(num_pages), _ptr(out["kv_indptr"]), _ptr(out["kv_indices"]), _ptr(out["kv_last_page_len"]),
        _ptr(out["qo_indptr"]), _ptr(out["slot_mapping"]), int(np.dtype(slot_dtype) == np.int64),
        kv_indices_capacity, slot_capacity, ctypes.addressof(err))
    out["kv_indices"] = out["kv_indices"][:kv_indices_capacity]
    out["kv_last_page_len"] = out["kv_last_page_len"][:B]
    out["slot_mapping"] = out["slot_mapping"][:slot_capacity]
    out["err"] = int(err.value)
    out["rc"] = int(rc)
    return out


def gather(indices: np.ndarray, table: np.ndarray, num_rows: int | None = None) -> tuple[np.ndarray, int]:
    """out[i] = table[indices[i]] (out-of-range rows zero); returns (out, error bits)."""
    assert table.ndim == 2 and table.strides[1] == table.itemsize
    idx = np.ascontiguousarray(indices)
    assert idx.dtype in (np.int32, np.int64) and idx.ndim == 1
    out = np.empty((idx.shape[0], table.shape[1]), table.dtype)
    err = ctypes.c_uint32(0)
    if idx.shape[0]:
        lib().oracle_gather_rows(_ptr(table), _ptr(out), _ptr(idx), int(idx.dtype == np.int64), idx.shape[0],
                                 table.shape[1] * table.itemsize, table.strides[0], out.strides[0],
                                 table.shape[0] if num_rows is None else num_rows, ctypes.addressof(err))
    return out, int(err.value)


def make_2d_indices(ranges, capacity: int | None = None) -> tuple[np.ndarray, int, int]:
    """Make2DIndices (batch_manager.h:30-51) over {row, col_start, col_end}
    ranges: returns (the first min(total, capacity) indices as int64, total,
    error bits); capacity None means room for all of them."""
    r = np.ascontiguousarray(np.asarray(ranges, np.int64).reshape(-1, 3))
    count = ctypes.c_int64(0)
    if capacity is None:
        lib().oracle_make_2d_indices(_ptr(r), r.shape[0], None, 0, ctypes.addressof(count))
        capacity = int(count.value)
    out = np.zeros(max(capacity, 1), np.int64)
    err = lib().oracle_make_2d_indices(_ptr(r), r.shape[0], _ptr(out), capacity, ctypes.addressof(count))
    total = int(count.value)
    return out[:min(total, capacity)].copy(), total, int(err)


class PagePool:
    """The free-page list of KVCacheManager (cache_manager.h:105-131) on the
    host: free_pages[:count] are free, the top is the end.  reserve/release
    update it and the int32 page table in place and return error bits."""

    def __init__(self, num_pages: int, free_pages: np.ndarray | None = None):
        self.capacity = num_pages
        self.free_pages = (np.arange(num_pages, dtype=np.int32) if free_pages is None
                           else np.ascontiguousarray(free_pages, np.int32).copy())
        self.count = np.array([self.free_pages.shape[0]], np.int32)
        self.free_pages = np.concatenate([self.free_pages, np.full(num_pages - self.free_pages.shape[0], -1,
                                                                   np.int32)])

    def reserve(self, table: np.ndarray, prior, new, page_size: int, table_index=None) -> int:
        assert table.dtype == np.int32 and table.flags.c_contiguous
        prior = np.ascontiguousarray(prior, np.int32)
        new = np.ascontiguousarray(new, np.int32)
        ti = None if table_index is None else np.ascontiguousarray(table_index, np.int32)
        return int(lib().oracle_reserve_pages(_ptr(self.free_pages), _ptr(self.count), self.capacity, _ptr(table),
                                              table.shape[1], table.shape[0], table.shape[1], _ptr(prior), _ptr(new),
                                              None if ti is None else _ptr(ti), page_size, prior.shape[0]))

    def release(self, table: np.ndarray, rows, num_tokens, page_size: int) -> int:
        rows = np.ascontiguousarray(rows, np.int32)
        toks = np.ascontiguousarray(num_tokens, np.int32)
        return int(lib().oracle_release_pages(_ptr(self.free_pages), _ptr(self.count), self.capacity, _ptr(table),
                                              table.shape[1], table.shape[0], table.shape[1], _ptr(rows), _ptr(toks),
                                              page_size, rows.shape[0]))

    def free_list(self) -> np.ndarray:
        return self.free_pages[:int(self.count[0])].copy()


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values rounded to bf16 or fp16 (round to nearest even), as float32."""
    x = np.asarray(x, np.float32)
    if dtype == "fp16":
        with np.errstate(over="ignore"):  # beyond fp16's range: inf, as the device conversion gives
            return x.astype(np.float16).astype(np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    r = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out)


def qkv_norm_rope_store(q, k, v, k_cache, v_cache, slots, q_weight=None, k_weight=None, eps=1e-6, cos_sin=None,
                        positions=None, interleaved=False, dtype="bf16", num_slots=None):
    """Restatement of the unfused sequence the fused kernel replaces:
    per-head RMSNorm (flashinfer::norm::QKRMSNorm as called at
    src/layers/rsm_norm.cu:49: fp32 sum of squares, x * rsqrt(ss / d + eps) * w,
    one rounding to the storage type), then the rotary embedding of
    apply_rope_with_cos_sin_cache (fp32, one rounding), then the store of
    store_kv_cache.cu:60-72.  Arrays are float32 holding values of the
    storage type: q [N, Hq, D], k/v [N, Hk, D], caches [S, Hk, D] (updated in
    place).  Returns (q_out, error bits); rows with a bad position stay
    unwritten (NaN in q_out)."""
    q, k, v = (np.asarray(a, np.float32) for a in (q, k, v))
    N, Hq, D = q.shape
    S = k_cache.shape[0] if num_slots is None else num_slots
    err = 0

    def norm(x, w):
        if w is None:
            return x
        ss = np.sum(x * x, axis=-1, dtype=np.float32, keepdims=True)
        r = (np.float32(1.0) / np.sqrt(ss / np.float32(D) + np.float32(eps))).astype(np.float32)
        return round_to(x * r * np.asarray(w, np.float32), dtype)

    def rope(x, cs):
        c, s = cs[:, None, : D // 2], cs[:, None, D // 2:]
        y = np.empty_like(x)
        if interleaved:
            a, b = x[..., 0::2], x[..., 1::2]
            y[..., 0::2] = a * c - b * s
            y[..., 1::2] = b * c + a * s
        else:
            a, b = x[..., : D // 2], x[..., D // 2:]
            y[..., : D // 2] = a * c - b * s
            y[..., D // 2:] = b * c + a * s
        return y

    qn, kn = norm(q, q_weight), norm(k, k_weight)
    ok = np.ones(N, bool)
    if cos_sin is not None:
        pos = np.asarray(positions, np.int64)
        ok = (pos >= 0) & (pos < cos_sin.shape[0])
        if not ok.all():
            err |= POSITION_RANGE
        cs = np.asarray(cos_sin, np.float32)[np.where(ok, pos, 0)]
        qn, kn = rope(qn, cs), rope(kn, cs)
    q_out = np.full_like(q, np.nan)
    q_out[ok] = round_to(qn[ok], dtype)
    kn = round_to(kn, dtype)
    for i in range(N):
        if not ok[i]:
            continue
        s_ = int(slots[i])
        if s_ < 0 or s_ >= S:
            if s_ != -1:
                err |= SLOT_RANGE
            continue
        k_cache[s_] = kn[i]
        v_cache[s_] = v[i]
    return q_out, err


# ---------------------------------------------------------------------------
# Pure-Python restatement (small cases only).
# ---------------------------------------------------------------------------
def py_store(k, v, k_cache, v_cache, slots) -> None:
    """Row-by-row copy, last writer wins: k_cache[l, slots[i]] = k[l, i]."""
    k3, v3, kc3, vc3 = _as3(k), _as3(v), _as3(k_cache), _as3(v_cache)
    for layer in range(k3.shape[0]):
        for i, s in enumerate(slots.tolist()):
            if s < 0:
                continue
            kc3[layer, s] = k3[layer, i]
            vc3[layer, s] = v3[layer, i]


def py_make_2d_indices(ranges) -> np.ndarray:
    """Make2DIndices as written (batch_manager.h:40-47), valid ranges only:
    row + start .. row + end - 1 for every range, in order."""
    out = []
    for row, start, end in np.asarray(ranges, np.int64).reshape(-1, 3).tolist():
        out += range(row + start, row + end)
    return np.array(out, np.int64)


def py_build_index(prior_len, new_len, page_table, page_size, table_index=None):
    """Straight loops over the formulas of the index contract (valid inputs)."""
    kv_indptr, kv_indices, last, qo_indptr, slots = [0], [], [], [0], []
    for i, (p, n) in enumerate(zip(list(prior_len), list(new_len))):
        row = i if table_index is None else int(table_index[i])
        total = int(p) + int(n)
        pages = -(-total // page_size)
        kv_indices += [int(x) for x in page_table[row][:pages]]
        kv_indptr.append(kv_indptr[-1] + pages)
        last.append(0 if total == 0 else (total - 1) % page_size + 1)
        qo_indptr.append(qo_indptr[-1] + int(n))
        for t in range(int(n)):
            pos = int(p) + t
            slots.append(int(page_table[row][pos // page_size]) * page_size + pos % page_size)
    return {
        "kv_indptr": np.array(kv_indptr, np.int32),
        "kv_indices": np.array(kv_indices, np.int32),
        "kv_last_page_len": np.array(last, np.int32),
        "qo_indptr": np.array(qo_indptr, np.int32),
        "slot_mapping": np.array(slots, np.int64),
    }


# ---------------------------------------------------------------------------
# libtorch restatement on CPU tensors: the reference's store and the index
# work of NextBatch expressed as libtorch CPU ops, which is how the reference's
# host code runs its tensor work.  The CPU baseline times it on all host
# threads; tests check it against the C oracle.
# ---------------------------------------------------------------------------
def torch_build_index(prior_len, new_len, page_table, page_size: int) -> dict:
    """The five index arrays of a batch with valid inputs (lengths >= 0, rows
    long enough) from int32 CPU tensors, vectorised over the batch: page
    counts and their cumulative sums (the per-request ranges of
    batch_manager.h:97-107), each sequence's page-table prefix (the load
    indices, :106) and the slots of its new tokens (out_loc, :109-110)."""
    import torch

    prior = prior_len.to(torch.int64).clamp(min=0)
    new = new_len.to(torch.int64).clamp(min=0)
    total = prior + new
    W = page_table.shape[1]
    pages = torch.clamp((total + page_size - 1) // page_size, max=W)
    zero = torch.zeros(1, dtype=torch.int64)
    kv_indptr = torch.cat([zero, pages.cumsum(0)])
    qo_indptr = torch.cat([zero, new.cumsum(0)])
    last = torch.where(pages == 0, torch.zeros_like(total), (total - 1) % page_size + 1)
    kv_indices = page_table[:prior.shape[0]][torch.arange(W)[None, :] < pages[:, None]]
    seq = torch.repeat_interleave(torch.arange(prior.shape[0]), new)
    pos = prior[seq] + torch.arange(seq.shape[0]) - qo_indptr[seq]
    slots = page_table[seq, pos // page_size].to(torch.int64) * page_size + pos % page_size
    return {"kv_indptr": kv_indptr.to(torch.int32), "kv_indices": kv_indices.to(torch.int32),
            "kv_last_page_len": last.to(torch.int32), "qo_indptr": qo_indptr.to(torch.int32), "slot_mapping": slots}


def torch_store(k, v, k_pool, v_pool, slots) -> None:
    """StoreKVCacheKernel's k_cache[idx[i]] = k[i] (store_kv_cache.cu:60-72)
    per layer, as MHAKVCache::StoreKV calls it (mha_kvcache.h:76-86), with
    libtorch's CPU index_copy_ on the [pages * page_size, row] pool views:
    k, v [L, N, E], pools [L, S, E], slots int64 [N]."""
    for layer in range(k.shape[0]):
        k_pool[layer].index_copy_(0, slots, k[layer])
        v_pool[layer].index_copy_(0, slots, v[layer])
