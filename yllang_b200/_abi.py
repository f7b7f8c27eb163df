"""ctypes binding of the C ABI in include/yl_kvpath.h (libyl_kvpath.so).

This is the binding a Python caller of the shared library would write; the
structures mirror the header field by field (tests/test_abi.py checks the
offsets against the C compiler's).  There is no fallback: if the library is
missing the import fails loudly.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libyl_kvpath.so")

YL_OK = 0
YL_ERR_NULL_ARG = -1
YL_ERR_BAD_SIZE = -2
YL_ERR_ALIGNMENT = -3
YL_ERR_UNSUPPORTED = -4
YL_ERR_CUDA = -5

DEVERR_SLOT_RANGE = 0x1
DEVERR_PAGE_RANGE = 0x2
DEVERR_ROW_OVERFLOW = 0x4
DEVERR_INDICES_CAP = 0x8
DEVERR_SLOTS_CAP = 0x10
DEVERR_NEGATIVE_LEN = 0x20
DEVERR_INDPTR_OVERFLOW = 0x40
DEVERR_TABLE_ROW = 0x80
DEVERR_TOKEN_COUNT = 0x100
DEVERR_TIMEOUT = 0x200
DEVERR_INDEX_RANGE = 0x400
DEVERR_POSITION_RANGE = 0x800
DEVERR_POOL_EMPTY = 0x1000
DEVERR_POOL_OVERFLOW = 0x2000
DEVERR_DUPLICATE_ROW = 0x4000

ABI_VERSION = 1

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64


class StoreArgs(ctypes.Structure):
    """struct yl_store_args."""

    _fields_ = [
        ("k", _vp),
        ("v", _vp),
        ("k_cache", _vp),
        ("v_cache", _vp),
        ("slots", _vp),
        ("slot_is_int64", _i32),
        ("num_layers", _i32),
        ("num_tokens", _i64),
        ("row_bytes", _i64),
        ("k_row_stride", _i64),
        ("v_row_stride", _i64),
        ("cache_row_stride", _i64),
        ("k_layer_stride", _i64),
        ("v_layer_stride", _i64),
        ("cache_layer_stride", _i64),
        ("num_slots", _i64),
        ("error_word", _vp),
    ]


class IndexArgs(ctypes.Structure):
    """struct yl_index_args."""

    _fields_ = [
        ("prior_len", _vp),
        ("new_len", _vp),
        ("page_table", _vp),
        ("table_index", _vp),
        ("page_table_stride", _i64),
        ("num_table_rows", _i32),
        ("max_pages_per_row", _i32),
        ("page_size", _i32),
        ("batch_size", _i32),
        ("slot_is_int64", _i32),
        ("num_pages", _i64),
        ("kv_indptr", _vp),
        ("kv_indices", _vp),
        ("kv_last_page_len", _vp),
        ("qo_indptr", _vp),
        ("slot_mapping", _vp),
        ("kv_indices_capacity", _i64),
        ("slot_capacity", _i64),
        ("error_word", _vp),
    ]


class StepArgs(ctypes.Structure):
    """struct yl_step_args."""

    _fields_ = [("index", IndexArgs), ("store", StoreArgs)]


class GatherArgs(ctypes.Structure):
    """struct yl_gather_args."""

    _fields_ = [
        ("table", _vp),
        ("out", _vp),
        ("indices", _vp),
        ("index_is_int64", _i32),
        ("reserved", _i32),
        ("num_indices", _i64),
        ("row_bytes", _i64),
        ("table_row_stride", _i64),
        ("out_row_stride", _i64),
        ("num_rows", _i64),
        ("error_word", _vp),
    ]


class QkvStoreArgs(ctypes.Structure):
    """struct yl_qkv_store_args."""

    _fields_ = [
        ("q", _vp),
        ("k", _vp),
        ("v", _vp),
        ("q_out", _vp),
        ("k_cache", _vp),
        ("v_cache", _vp),
        ("slots", _vp),
        ("q_weight", _vp),
        ("k_weight", _vp),
        ("cos_sin_cache", _vp),
        ("positions", _vp),
        ("dtype", _i32),
        ("slot_is_int64", _i32),
        ("position_is_int64", _i32),
        ("rope_interleaved", _i32),
        ("num_q_heads", _i32),
        ("num_kv_heads", _i32),
        ("head_dim", _i32),
        ("eps", ctypes.c_float),
        ("num_tokens", _i64),
        ("q_row_stride", _i64),
        ("k_row_stride", _i64),
        ("v_row_stride", _i64),
        ("q_out_row_stride", _i64),
        ("cache_row_stride", _i64),
        ("num_slots", _i64),
        ("max_position", _i64),
        ("error_word", _vp),
    ]


YL_DTYPE_BF16, YL_DTYPE_F16 = 0, 1


def deverr_names(bits: int) -> str:
    """'SLOT_RANGE|PAGE_RANGE' for a device error word (YL_DEVERR_* bits)."""
    names = []
    for name, value in globals().items():
        if name.startswith("DEVERR_") and bits & value:
            names.append(name[len("DEVERR_"):])
            bits &= ~value
    if bits:
        names.append(hex(bits))
    return "|".join(names)


class PagePool(ctypes.Structure):
    """struct yl_page_pool."""

    _fields_ = [("free_pages", _vp), ("free_count", _vp), ("capacity", _i64)]


class ReserveArgs(ctypes.Structure):
    """struct yl_reserve_args."""

    _fields_ = [
        ("pool", PagePool),
        ("page_table", _vp),
        ("prior_len", _vp),
        ("new_len", _vp),
        ("table_index", _vp),
        ("page_table_stride", _i64),
        ("num_table_rows", _i32),
        ("max_pages_per_row", _i32),
        ("page_size", _i32),
        ("batch_size", _i32),
        ("error_word", _vp),
    ]


class ReleaseArgs(ctypes.Structure):
    """struct yl_release_args."""

    _fields_ = [
        ("pool", PagePool),
        ("page_table", _vp),
        ("rows", _vp),
        ("num_tokens", _vp),
        ("page_table_stride", _i64),
        ("num_table_rows", _i32),
        ("max_pages_per_row", _i32),
        ("page_size", _i32),
        ("num_release", _i32),
        ("error_word", _vp),
    ]


class RangesArgs(ctypes.Structure):
    """struct yl_ranges_args."""

    _fields_ = [
        ("ranges", _vp),
        ("indices", _vp),
        ("count", _vp),
        ("num_ranges", _i64),
        ("indices_capacity", _i64),
        ("error_word", _vp),
    ]


# Every symbol include/yl_kvpath.h declares.
EXPORTED_SYMBOLS = ("yl_kv_store", "yl_build_index", "yl_kv_step", "yl_gather_rows", "yl_qkv_norm_rope_store",
                    "yl_reserve_pages", "yl_release_pages", "yl_make_2d_indices", "yl_status_string", "yl_last_error",
                    "yl_abi_version")

_lib: ctypes.CDLL | None = None


class KVPathError(RuntimeError):
    """A yl_* entry point returned a negative status."""

    def __init__(self, status: int, detail: str):
        super().__init__(f"{status_string(status)} ({status}): {detail}")
        self.status = status
        self.detail = detail


def lib() -> ctypes.CDLL:
    """Load libyl_kvpath.so (built in-tree by __graft_entry__.build())."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build the CUDA library first "
                              "(python -c 'import __graft_entry__ as g; g.build()')")
        L = ctypes.CDLL(LIB_PATH)
        L.yl_kv_store.restype = ctypes.c_int
        L.yl_kv_store.argtypes = [ctypes.POINTER(StoreArgs), _vp]
        L.yl_build_index.restype = ctypes.c_int
        L.yl_build_index.argtypes = [ctypes.POINTER(IndexArgs), _vp]
        L.yl_kv_step.restype = ctypes.c_int
        L.yl_kv_step.argtypes = [ctypes.POINTER(StepArgs), _vp]
        L.yl_gather_rows.restype = ctypes.c_int
        L.yl_gather_rows.argtypes = [ctypes.POINTER(GatherArgs), _vp]
        L.yl_qkv_norm_rope_store.restype = ctypes.c_int
        L.yl_qkv_norm_rope_store.argtypes = [ctypes.POINTER(QkvStoreArgs), _vp]
        L.yl_reserve_pages.restype = ctypes.c_int
        L.yl_reserve_pages.argtypes = [ctypes.POINTER(ReserveArgs), _vp]
        L.yl_release_pages.restype = ctypes.c_int
        L.yl_release_pages.argtypes = [ctypes.POINTER(ReleaseArgs), _vp]
        L.yl_make_2d_indices.restype = ctypes.c_int
        L.yl_make_2d_indices.argtypes = [ctypes.POINTER(RangesArgs), _vp]
        L.yl_status_string.restype = ctypes.c_char_p
        L.yl_status_string.argtypes = [ctypes.c_int]
        L.yl_last_error.restype = ctypes.c_char_p
        L.yl_last_error.argtypes = []
        L.yl_abi_version.restype = ctypes.c_int
        L.yl_abi_version.argtypes = []
        if L.yl_abi_version() != ABI_VERSION:
            raise ImportError(f"libyl_kvpath.so ABI {L.yl_abi_version()} != binding ABI {ABI_VERSION}")
        _lib = L
    return _lib


def status_string(status: int) -> str:
    return lib().yl_status_string(status).decode()


def last_error() -> str:
    return lib().yl_last_error().decode()


def check(status: int) -> None:
    if status != YL_OK:
        raise KVPathError(status, last_error())


def kv_store_raw(args: StoreArgs, stream: int | None) -> int:
    return lib().yl_kv_store(ctypes.byref(args), stream)


def build_index_raw(args: IndexArgs, stream: int | None) -> int:
    return lib().yl_build_index(ctypes.byref(args), stream)


def kv_step_raw(args: StepArgs, stream: int | None) -> int:
    return lib().yl_kv_step(ctypes.byref(args), stream)


def gather_rows_raw(args: GatherArgs, stream: int | None) -> int:
    return lib().yl_gather_rows(ctypes.byref(args), stream)


def qkv_store_raw(args: QkvStoreArgs, stream: int | None) -> int:
    return lib().yl_qkv_norm_rope_store(ctypes.byref(args), stream)


def reserve_pages_raw(args: ReserveArgs, stream: int | None) -> int:
    return lib().yl_reserve_pages(ctypes.byref(args), stream)


def release_pages_raw(args: ReleaseArgs, stream: int | None) -> int:
    return lib().yl_release_pages(ctypes.byref(args), stream)


def make_2d_indices_raw(args: RangesArgs, stream: int | None) -> int:
    return lib().yl_make_2d_indices(ctypes.byref(args), stream)
