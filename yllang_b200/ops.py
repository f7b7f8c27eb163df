"""Torch-tensor front end of the C ABI, for Python callers, tests and the bench.

Each function checks its tensors the way the reference's TensorMatcher does
for StoreKVCache (src/kvcache/store_kv_cache.cu:108-124: caches [*, E] with
stride [cs, 1], inputs [N, E] with stride [ks, 1], indices [N] with stride
[1], one device, one dtype), turns them into the raw pointers and byte
strides of yl_store_args / yl_index_args, and calls libyl_kvpath.so on the
current CUDA stream.  A contract violation raises PanicError before any
launch, as RuntimeCheck does in the reference (src/include/util/panic.h:35).
"""
from __future__ import annotations

import os
from typing import NamedTuple

import torch

from . import _abi


class PanicError(RuntimeError):
    """Contract violation detected on the host (yllang::PanicError)."""


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise PanicError(msg)


# Debug mode, off by default: YLLANG_CHECK_DEVICE_ERRORS=1 in the environment
# (read at import).  A call given no device error word then runs its kernels
# with a private one, waits for it and raises PanicError naming the bits they
# raised (the check of what the kernels otherwise skip and only flag).  Every
# such call becomes synchronous, so it cannot be captured in a CUDA graph.
CHECK_DEVICE_ERRORS = os.environ.get("YLLANG_CHECK_DEVICE_ERRORS", "") not in ("", "0")


def _word(error_word: torch.Tensor | None, device: torch.device, what: str) -> int | None:
    """Device pointer of a caller's error word: a 4-byte tensor on `device`."""
    if error_word is None:
        return None
    _check(error_word.is_cuda and error_word.device == device and error_word.element_size() == 4
           and error_word.numel() >= 1, f"{what}: error_word must be a 4-byte tensor on {device}")
    return error_word.data_ptr()


class _Errors:
    """The error word of one call: the caller's, or in debug mode a private
    one that check() reads back after the launch.  The private word is zeroed
    on the call's stream and read after that stream has finished, so a call
    on a side stream is checked like one on the current stream."""

    def __init__(self, error_word: torch.Tensor | None, device: torch.device, what: str,
                 stream: torch.cuda.Stream | None = None):
        self.what = what
        self.private = None
        self.tensor = error_word
        if error_word is None and CHECK_DEVICE_ERRORS:
            self.stream = stream if stream is not None else torch.cuda.current_stream(device)
            with torch.cuda.stream(self.stream):
                self.private = self.tensor = torch.zeros(1, dtype=torch.int32, device=device)
        self.ptr = _word(self.tensor, device, what)

    def check(self) -> None:
        if self.private is not None:
            self.stream.synchronize()
            bits = int(self.private.item()) & 0xFFFFFFFF
            if bits:
                raise PanicError(f"{self.what}: device error bits {bits:#x} ({_abi.deverr_names(bits)})")


def _stream(stream: torch.cuda.Stream | None, device: torch.device) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return s.cuda_stream


def store_args(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
               slots: torch.Tensor, error_word: torch.Tensor | None = None,
               check_slots: bool = True) -> _abi.StoreArgs:
    """Validate and pack one store call.

    Per-layer form (the reference's): k, v [N, E]; k_cache, v_cache [S, E].
    All-layers form: k, v [L, N, E]; k_cache, v_cache [L, S, E].
    """
    _check(k.dim() in (2, 3), f"k must be [N, E] or [L, N, E], got {tuple(k.shape)}")
    multi = k.dim() == 3
    for name, t in (("v", v), ("k_cache", k_cache), ("v_cache", v_cache)):
        _check(t.dim() == k.dim(), f"{name} rank {t.dim()} != k rank {k.dim()}")
    _check(k.shape == v.shape, f"v shape {tuple(v.shape)} != k shape {tuple(k.shape)}")
    _check(k_cache.shape == v_cache.shape, "k_cache and v_cache shapes differ")
    _check(k_cache.stride() == v_cache.stride(), "k_cache and v_cache strides differ")
    E = k.shape[-1]
    _check(k_cache.shape[-1] == E, f"cache row {k_cache.shape[-1]} != input row {E}")
    if multi:
        _check(k_cache.shape[0] == k.shape[0], "layer counts of inputs and caches differ")
    for name, t in (("k", k), ("v", v), ("k_cache", k_cache), ("v_cache", v_cache)):
        _check(t.stride(-1) == 1, f"{name} rows must be contiguous (stride[-1] == 1)")
        _check(t.dtype == k.dtype, f"{name} dtype {t.dtype} != {k.dtype}")
        _check(t.device == k.device, f"{name} on {t.device}, expected {k.device}")
    _check(k.is_cuda, "tensors must be CUDA tensors")
    N = k.shape[-2]
    _check(slots.dim() == 1 and slots.shape[0] == N, f"slots must be [N={N}], got {tuple(slots.shape)}")
    _check(slots.stride(0) == 1 or N <= 1, "slots must be contiguous")
    _check(slots.dtype in (torch.int32, torch.int64), f"slots dtype {slots.dtype} must be int32 or int64")
    _check(slots.device == k.device, "slots on another device")
    item = k.element_size()
    a = _abi.StoreArgs()
    a.k, a.v = k.data_ptr(), v.data_ptr()
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.slots = slots.data_ptr()
    a.slot_is_int64 = int(slots.dtype == torch.int64)
    a.num_layers = k.shape[0] if multi else 1
    a.num_tokens = N
    a.row_bytes = E * item
    a.k_row_stride = k.stride(-2) * item
    a.v_row_stride = v.stride(-2) * item
    a.cache_row_stride = k_cache.stride(-2) * item
    if multi:
        a.k_layer_stride = k.stride(0) * item
        a.v_layer_stride = v.stride(0) * item
        a.cache_layer_stride = k_cache.stride(0) * item
    a.num_slots = k_cache.shape[-2] if check_slots else 0
    a.error_word = _word(error_word, k.device, "store")
    return a


def store_kv_cache(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                   slots: torch.Tensor, error_word: torch.Tensor | None = None,
                   stream: torch.cuda.Stream | None = None) -> None:
    """k_cache[..., slots[i], :] = k[..., i, :] (and v), asynchronously.

    Mirrors yllang::StoreKVCache (src/kvcache/store_kv_cache.cu:95-163) with
    the row size taken at run time; a [L, N, E] input stores all L layers in
    one launch.
    """
    if k.shape[-2] == 0:
        return
    errs = _Errors(error_word, k.device, "store_kv_cache", stream)
    args = store_args(k, v, k_cache, v_cache, slots, errs.tensor)
    _abi.check(_abi.kv_store_raw(args, _stream(stream, k.device)))
    errs.check()


class BatchIndex(NamedTuple):
    """Page arrays of one batch, in the paged-KV format of flashinfer."""

    kv_indptr: torch.Tensor
    kv_indices: torch.Tensor
    kv_last_page_len: torch.Tensor
    qo_indptr: torch.Tensor
    slot_mapping: torch.Tensor


def _check_index_inputs(prior_len, new_len, page_table, table_index) -> None:
    dev = prior_len.device
    _check(prior_len.is_cuda, "prior_len must be a CUDA tensor")
    for name, t in (("prior_len", prior_len), ("new_len", new_len), ("page_table", page_table)):
        _check(t.dtype == torch.int32, f"{name} must be int32, got {t.dtype}")
        _check(t.device == dev, f"{name} on {t.device}, expected {dev}")
    B = prior_len.shape[0]
    _check(prior_len.dim() == 1 and new_len.shape == (B,), "prior_len and new_len must both be [B]")
    _check(prior_len.is_contiguous() and new_len.is_contiguous(), "lengths must be contiguous")
    _check(page_table.dim() == 2 and page_table.stride(1) == 1, "page_table must be [R, W] with unit column stride")
    if table_index is not None:
        _check(table_index.dtype == torch.int32 and table_index.shape == (B,) and table_index.is_contiguous()
               and table_index.device == dev, "table_index must be contiguous int32 [B] on the same device")
    else:
        _check(page_table.shape[0] >= B, f"page_table has {page_table.shape[0]} rows for a batch of {B}")


def _check_out(out: "BatchIndex", B: int, dev) -> None:
    for name in ("kv_indptr", "kv_indices", "kv_last_page_len", "qo_indptr"):
        t = getattr(out, name)
        _check(t.dtype == torch.int32 and t.device == dev and t.is_contiguous(), f"out.{name}: contiguous int32")
    _check(out.kv_indptr.numel() >= B + 1 and out.qo_indptr.numel() >= B + 1, "out indptrs need B + 1 entries")
    _check(out.kv_last_page_len.numel() >= B, "out.kv_last_page_len needs B entries")
    _check(out.slot_mapping.dtype in (torch.int32, torch.int64) and out.slot_mapping.is_contiguous()
           and out.slot_mapping.device == dev, "out.slot_mapping: contiguous int32 or int64")


def build_index(prior_len: torch.Tensor, new_len: torch.Tensor, page_table: torch.Tensor, page_size: int,
                table_index: torch.Tensor | None = None, num_pages: int = 0, kv_indices_capacity: int | None = None,
                slot_capacity: int | None = None, slot_dtype: torch.dtype = torch.int64,
                error_word: torch.Tensor | None = None, out: BatchIndex | None = None,
                stream: torch.cuda.Stream | None = None) -> BatchIndex:
    """Build kv_indptr / kv_indices / kv_last_page_len / qo_indptr / slot_mapping.

    prior_len, new_len: int32 [B] on the device.  page_table: int32 [R, W]
    with unit column stride.  The capacities bound the two ragged outputs;
    when omitted they are computed from the lengths, which costs a device to
    host read (pass them, or `out`, on a hot path).
    """
    _check_index_inputs(prior_len, new_len, page_table, table_index)
    dev = prior_len.device
    B = prior_len.shape[0]
    W = page_table.shape[1]
    if out is None:
        _check(slot_dtype in (torch.int32, torch.int64), "slot_dtype must be int32 or int64")
        if kv_indices_capacity is None or slot_capacity is None:
            tot = prior_len.clamp(min=0).to(torch.int64) + new_len.clamp(min=0).to(torch.int64)
            if kv_indices_capacity is None:
                kv_indices_capacity = int(torch.clamp((tot + page_size - 1) // page_size, max=W).sum())
            if slot_capacity is None:
                slot_capacity = int(new_len.clamp(min=0).to(torch.int64).sum())
        i32 = dict(dtype=torch.int32, device=dev)
        out = BatchIndex(torch.empty(B + 1, **i32), torch.empty(kv_indices_capacity, **i32),
                         torch.empty(B, **i32), torch.empty(B + 1, **i32),
                         torch.empty(slot_capacity, dtype=slot_dtype, device=dev))
    _check_out(out, B, dev)
    errs = _Errors(error_word, dev, "build_index", stream)
    a = index_args(prior_len, new_len, page_table, page_size, table_index, num_pages, out, errs.tensor)
    _abi.check(_abi.build_index_raw(a, _stream(stream, dev)))
    errs.check()
    return out


def index_args(prior_len, new_len, page_table, page_size, table_index, num_pages, out: BatchIndex,
               error_word) -> _abi.IndexArgs:
    """Pack validated index tensors into yl_index_args."""
    a = _abi.IndexArgs()
    a.prior_len, a.new_len = prior_len.data_ptr(), new_len.data_ptr()
    a.page_table = page_table.data_ptr()
    a.table_index = table_index.data_ptr() if table_index is not None else None
    a.page_table_stride = page_table.stride(0)
    a.num_table_rows = page_table.shape[0]
    a.max_pages_per_row = page_table.shape[1]
    a.page_size = page_size
    a.batch_size = prior_len.shape[0]
    a.slot_is_int64 = int(out.slot_mapping.dtype == torch.int64)
    a.num_pages = num_pages
    a.kv_indptr, a.kv_indices = out.kv_indptr.data_ptr(), out.kv_indices.data_ptr()
    a.kv_last_page_len, a.qo_indptr = out.kv_last_page_len.data_ptr(), out.qo_indptr.data_ptr()
    a.slot_mapping = out.slot_mapping.data_ptr()
    a.kv_indices_capacity = out.kv_indices.numel()
    a.slot_capacity = out.slot_mapping.numel()
    a.error_word = _word(error_word, prior_len.device, "index")
    return a


def kv_step(prior_len: torch.Tensor, new_len: torch.Tensor, page_table: torch.Tensor, page_size: int,
            k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, out: BatchIndex,
            table_index: torch.Tensor | None = None, num_pages: int = 0, error_word: torch.Tensor | None = None,
            stream: torch.cuda.Stream | None = None) -> BatchIndex:
    """One step: build_index(...) into `out`, then store_kv_cache(k, v,
    k_cache, v_cache, out.slot_mapping), fused into one launch (yl_kv_step).

    k, v are [N, E] (one layer) or [L, N, E] (every layer); k_cache, v_cache
    the matching per-layer [S, E] or all-layer [L, S, E] pool views; N must
    equal the sum of new_len.  `out` must have room for the batch's pages and
    at least N slots (its slot dtype decides the slot type).
    """
    _check(out is not None, "kv_step needs preallocated outputs (out=)")
    _check_index_inputs(prior_len, new_len, page_table, table_index)
    _check_out(out, prior_len.shape[0], prior_len.device)
    N = k.shape[-2]
    _check(out.slot_mapping.numel() >= N, f"out.slot_mapping holds {out.slot_mapping.numel()} < N={N} slots")
    a = _abi.StepArgs()
    a.store = store_args(k, v, k_cache, v_cache, out.slot_mapping[:N], None)
    errs = _Errors(error_word, prior_len.device, "kv_step", stream)  # the step reports store errors here too
    a.index = index_args(prior_len, new_len, page_table, page_size, table_index, num_pages, out, errs.tensor)
    _abi.check(_abi.kv_step_raw(a, _stream(stream, k.device)))
    errs.check()
    return out


def gather_rows(indices: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None,
                error_word: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """out[i, :] = table[indices[i], :] (the embedding lookup); rows whose index
    is outside the table come out zero (-1 silently, others also set
    DEVERR_INDEX_RANGE).  Mirrors yllang::Index (src/layers/index.cu:93-146)
    with the contract its TensorMatcher enforces (index.cu:104-119)."""
    _check(table.dim() == 2 and table.stride(1) == 1, "table must be [V, E] with contiguous rows")
    _check(table.is_cuda, "table must be a CUDA tensor")
    _check(indices.dim() == 1 and (indices.stride(0) == 1 or indices.numel() <= 1), "indices must be [N], contiguous")
    _check(indices.dtype in (torch.int32, torch.int64), "indices must be int32 or int64")
    _check(indices.device == table.device, "indices on another device")
    N, E = indices.shape[0], table.shape[1]
    if out is None:
        out = torch.empty(N, E, dtype=table.dtype, device=table.device)
    _check(out.dim() == 2 and out.shape == (N, E) and out.stride(1) == 1, f"out must be [{N}, {E}] with contiguous rows")
    _check(out.dtype == table.dtype and out.device == table.device, "out dtype/device must match the table")
    if N == 0:
        return out
    item = table.element_size()
    a = _abi.GatherArgs()
    a.table, a.out, a.indices = table.data_ptr(), out.data_ptr(), indices.data_ptr()
    a.index_is_int64 = int(indices.dtype == torch.int64)
    a.num_indices = N
    a.row_bytes = E * item
    a.table_row_stride = table.stride(0) * item
    a.out_row_stride = out.stride(0) * item
    a.num_rows = table.shape[0]
    errs = _Errors(error_word, table.device, "gather_rows", stream)
    a.error_word = errs.ptr
    _abi.check(_abi.gather_rows_raw(a, _stream(stream, table.device)))
    errs.check()
    return out


def make_2d_indices(ranges: torch.Tensor, out: torch.Tensor | None = None, count: torch.Tensor | None = None,
                    error_word: torch.Tensor | None = None,
                    stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Flat indices of {row, col_start, col_end} ranges: row + c for c in
    [col_start, col_end), range after range (Make2DIndices,
    src/include/batch/batch_manager.h:30-51, as int64 instead of float).

    ranges: device int64 [R, 3].  With ``out`` (device int64 [capacity]) the
    call never leaves the device: indices past the capacity are dropped and
    flagged (DEVERR_INDICES_CAP), and ``count`` (device int64 [1]) receives the
    total.  Without ``out`` the total is computed here from the ranges (one
    copy to the host), invalid ranges raise PanicError, and a tensor of exactly
    that length is returned."""
    _check(ranges.is_cuda, "ranges must be a CUDA tensor")
    _check(ranges.dtype == torch.int64, f"ranges dtype {ranges.dtype} must be int64")
    _check(ranges.dim() == 2 and ranges.shape[1] == 3, f"ranges must be [R, 3], got {tuple(ranges.shape)}")
    _check(ranges.is_contiguous(), "ranges must be contiguous")
    dev = ranges.device
    if out is None:
        if stream is not None:
            stream.synchronize()  # the ranges may come from work on the call's stream
        host = ranges.cpu()
        row, lo, hi = host[:, 0], host[:, 1], host[:, 2]
        _check(bool((row >= 0).all() and (lo >= 0).all() and (hi >= lo).all()),
               "ranges need row >= 0, col_start >= 0 and col_end >= col_start")
        _check(all(r <= (1 << 63) - 1 - h for r, h in zip(row.tolist(), hi.tolist())),
               "ranges: row + col_end passes INT64_MAX")
        total = sum((hi - lo).tolist())
        _check(total < (1 << 40), f"ranges: {total} indices is not below 2^40")
        with torch.cuda.stream(stream if stream is not None else torch.cuda.current_stream(dev)):
            out = torch.empty(total, dtype=torch.int64, device=dev)  # owned by the stream that writes it
    _check(out.dtype == torch.int64 and out.dim() == 1 and out.is_contiguous() and out.device == dev,
           "out must be a contiguous int64 [capacity] tensor on the ranges' device")
    if count is not None:
        _check(count.dtype == torch.int64 and count.numel() >= 1 and count.device == dev,
               "count must be an int64 tensor on the ranges' device")
    a = _abi.RangesArgs()
    a.ranges = ranges.data_ptr() if ranges.numel() else None
    a.indices = out.data_ptr() if out.numel() else None
    a.count = count.data_ptr() if count is not None else None
    a.num_ranges = ranges.shape[0]
    a.indices_capacity = out.numel()
    errs = _Errors(error_word, dev, "make_2d_indices", stream)
    a.error_word = errs.ptr
    _abi.check(_abi.make_2d_indices_raw(a, _stream(stream, dev)))
    errs.check()
    return out


def rope_cos_sin_cache(max_position: int, head_dim: int, theta: float = 1e6,
                       device: torch.device | str = "cpu") -> torch.Tensor:
    """[max_position, head_dim] fp32: head_dim / 2 cosines then head_dim / 2
    sines of p * theta^(-2j / head_dim) (the model config's rope_theta,
    src/models/model_config.cpp:38; 1e6 for Qwen3)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    angles = torch.arange(max_position, dtype=torch.float64)[:, None] * inv_freq[None, :]
    return torch.cat([angles.cos(), angles.sin()], dim=1).to(torch.float32).to(device).contiguous()


def _heads(t: torch.Tensor, name: str) -> tuple[int, int]:
    _check(t.dim() == 3 and t.stride(2) == 1 and t.stride(1) == t.shape[2], f"{name} must be [N, heads, head_dim] "
           "with contiguous heads")
    return t.shape[1], t.shape[2]


def qkv_norm_rope_store(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                        v_cache: torch.Tensor, slots: torch.Tensor, *, q_weight: torch.Tensor | None = None,
                        k_weight: torch.Tensor | None = None, eps: float = 1e-6,
                        cos_sin_cache: torch.Tensor | None = None, positions: torch.Tensor | None = None,
                        interleaved: bool = False, q_out: torch.Tensor | None = None,
                        error_word: torch.Tensor | None = None,
                        stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """One layer's attention input in one launch: per-head RMSNorm of q and k
    (weights [head_dim]; None skips it), rotary embedding by positions from
    cos_sin_cache (None skips it), then q written to q_out (default: a new
    tensor; q itself for in place) and k, v stored into the pool rows
    k_cache[slots[i]], v_cache[slots[i]].

    q [N, Hq, D], k/v [N, Hk, D] (token rows may be strided, e.g. views of
    one fused QKV projection); k_cache/v_cache [S, Hk * D] pool rows; slots
    and positions int32 or int64 [N].  Returns q_out."""
    Hq, D = _heads(q, "q")
    Hk, Dk = _heads(k, "k")
    _check(Dk == D and tuple(v.shape) == tuple(k.shape) and v.stride(2) == 1 and v.stride(1) == D,
           "k and v must be [N, Hk, head_dim] with the head_dim of q")
    N = q.shape[0]
    _check(k.shape[0] == N and slots.dim() == 1 and slots.shape[0] == N, "q, k, v and slots must have N rows")
    _check(q.dtype in (torch.bfloat16, torch.float16), "q/k/v must be bf16 or fp16")
    for name, t in (("k", k), ("v", v), ("k_cache", k_cache), ("v_cache", v_cache)):
        _check(t.dtype == q.dtype and t.device == q.device, f"{name} dtype/device must match q")
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache)):
        _check(t.dim() == 2 and t.shape[1] == Hk * D and t.stride(1) == 1, f"{name} must be [S, {Hk * D}] pool rows")
    _check(k_cache.shape == v_cache.shape and k_cache.stride(0) == v_cache.stride(0),
           "k_cache and v_cache must share shape and row stride")
    _check(q.is_cuda, "q must be a CUDA tensor")
    _check(slots.dtype in (torch.int32, torch.int64) and slots.device == q.device and (slots.stride(0) == 1 or N <= 1),
           "slots must be contiguous int32/int64 on q's device")
    for name, w in (("q_weight", q_weight), ("k_weight", k_weight)):
        _check(w is None or (w.shape == (D,) and w.dtype == q.dtype and w.device == q.device and w.is_contiguous()),
               f"{name} must be [{D}] of q's dtype and device")
    if cos_sin_cache is not None:
        _check(cos_sin_cache.dim() == 2 and cos_sin_cache.shape[1] == D and cos_sin_cache.dtype == torch.float32
               and cos_sin_cache.is_contiguous() and cos_sin_cache.device == q.device,
               f"cos_sin_cache must be contiguous fp32 [max_position, {D}] on q's device")
        _check(positions is not None and positions.dim() == 1 and positions.shape[0] == N
               and positions.dtype in (torch.int32, torch.int64) and positions.device == q.device
               and (positions.stride(0) == 1 or N <= 1), "positions must be contiguous int32/int64 [N]")
    if q_out is None:
        q_out = torch.empty(N, Hq, D, dtype=q.dtype, device=q.device)
    _check(q_out.shape == q.shape and q_out.dtype == q.dtype and q_out.stride(2) == 1 and q_out.stride(1) == D,
           "q_out must be [N, Hq, head_dim] like q")
    item = q.element_size()
    a = _abi.QkvStoreArgs()
    a.q, a.k, a.v, a.q_out = q.data_ptr(), k.data_ptr(), v.data_ptr(), q_out.data_ptr()
    a.k_cache, a.v_cache, a.slots = k_cache.data_ptr(), v_cache.data_ptr(), slots.data_ptr()
    a.q_weight = q_weight.data_ptr() if q_weight is not None else None
    a.k_weight = k_weight.data_ptr() if k_weight is not None else None
    if cos_sin_cache is not None:
        a.cos_sin_cache, a.positions = cos_sin_cache.data_ptr(), positions.data_ptr()
        a.position_is_int64 = int(positions.dtype == torch.int64)
        a.max_position = cos_sin_cache.shape[0]
    a.dtype = _abi.YL_DTYPE_BF16 if q.dtype == torch.bfloat16 else _abi.YL_DTYPE_F16
    a.slot_is_int64 = int(slots.dtype == torch.int64)
    a.rope_interleaved = int(bool(interleaved))
    a.num_q_heads, a.num_kv_heads, a.head_dim, a.eps = Hq, Hk, D, float(eps)
    a.num_tokens = N
    a.q_row_stride, a.k_row_stride, a.v_row_stride = q.stride(0) * item, k.stride(0) * item, v.stride(0) * item
    a.q_out_row_stride = q_out.stride(0) * item
    a.cache_row_stride = k_cache.stride(0) * item
    a.num_slots = k_cache.shape[0]
    errs = _Errors(error_word, q.device, "qkv_norm_rope_store", stream)
    a.error_word = errs.ptr
    _abi.check(_abi.qkv_store_raw(a, _stream(stream, q.device)))
    errs.check()
    return q_out


class DevicePagePool:
    """KVCacheManager's free-page list kept on the device (yl_reserve_pages /
    yl_release_pages): free_pages[:free_count] are the free page ids, the top
    of the stack is the end.  The initial list is page ids 0..num_pages-1 in
    order (the reference builds it with torch::range, cache_manager.h:33-34),
    unless `free_pages` gives another order.  All methods are asynchronous on
    the current stream except free_count()."""

    def __init__(self, num_pages: int, device: torch.device | str = "cuda", free_pages: torch.Tensor | None = None):
        _check(0 < num_pages < (1 << 31), "num_pages must be in [1, 2^31)")
        self.capacity = int(num_pages)
        self.device = torch.device(device)
        self.free_pages = torch.full((num_pages,), -1, dtype=torch.int32, device=self.device)
        init = torch.arange(num_pages, dtype=torch.int32) if free_pages is None else free_pages.to(torch.int32)
        _check(init.dim() == 1 and init.shape[0] <= num_pages, "free_pages must be [<= num_pages]")
        self.free_pages[:init.shape[0]].copy_(init)
        self.count = torch.tensor([init.shape[0]], dtype=torch.int32, device=self.device)

    def _pool(self) -> _abi.PagePool:
        return _abi.PagePool(self.free_pages.data_ptr(), self.count.data_ptr(), self.capacity)

    @staticmethod
    def _table(page_table: torch.Tensor):
        _check(page_table.dim() == 2 and page_table.dtype == torch.int32 and page_table.stride(1) == 1,
               "page_table must be int32 [rows, width] with unit column stride")
        return page_table.data_ptr(), page_table.stride(0), page_table.shape[0], page_table.shape[1]

    def _vec(self, t: torch.Tensor, n: int, name: str) -> int:
        _check(t.dim() == 1 and t.shape[0] == n and t.dtype == torch.int32 and t.device == self.device
               and (t.stride(0) == 1 or n <= 1), f"{name} must be contiguous int32 [{n}] on the pool's device")
        return t.data_ptr()

    def reserve(self, page_table: torch.Tensor, prior_len: torch.Tensor, new_len: torch.Tensor, page_size: int,
                table_index: torch.Tensor | None = None, error_word: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> None:
        """Give each sequence the pages its prior_len + new_len tokens lack,
        written into its page-table row (row table_index[i], default i)."""
        B = prior_len.shape[0]
        a = _abi.ReserveArgs()
        a.pool = self._pool()
        a.page_table, a.page_table_stride, a.num_table_rows, a.max_pages_per_row = self._table(page_table)
        a.prior_len = self._vec(prior_len, B, "prior_len")
        a.new_len = self._vec(new_len, B, "new_len")
        a.table_index = self._vec(table_index, B, "table_index") if table_index is not None else None
        a.page_size, a.batch_size = page_size, B
        errs = _Errors(error_word, self.device, "DevicePagePool.reserve", stream)
        a.error_word = errs.ptr
        _abi.check(_abi.reserve_pages_raw(a, _stream(stream, self.device)))
        errs.check()

    def release(self, page_table: torch.Tensor, rows: torch.Tensor, num_tokens: torch.Tensor, page_size: int,
                error_word: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> None:
        """Return the pages of each row (ceil(num_tokens / page_size)) to the
        list, in row order, and clear those table entries to -1."""
        R = rows.shape[0]
        a = _abi.ReleaseArgs()
        a.pool = self._pool()
        a.page_table, a.page_table_stride, a.num_table_rows, a.max_pages_per_row = self._table(page_table)
        a.rows = self._vec(rows, R, "rows")
        a.num_tokens = self._vec(num_tokens, R, "num_tokens")
        a.page_size, a.num_release = page_size, R
        errs = _Errors(error_word, self.device, "DevicePagePool.release", stream)
        a.error_word = errs.ptr
        _abi.check(_abi.release_pages_raw(a, _stream(stream, self.device)))
        errs.check()

    def free_count(self) -> int:
        return int(self.count.item())

    def free_list(self) -> torch.Tensor:
        return self.free_pages[:self.free_count()].clone()
