"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, its structs match the ctypes binding byte for byte, argument
errors come back as status codes before any launch, and the multiply-shift
divider used by the kernels is exact."""
import ctypes
import os
import re
import subprocess
import sys

import pytest

import yllang_b200 as yl
from yllang_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "yl_kvpath.h")


def _declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"YL_API\s+[\w\s\*]*?\b(yl_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = yl.lib()
    declared = _declared_symbols()
    assert declared == sorted(_abi.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _abi.LIB_PATH], capture_output=True, text=True, check=True)
    exported = sorted(set(re.findall(r" T (yl_\w+)", out.stdout)))
    assert exported == declared
    assert L.yl_abi_version() == _abi.ABI_VERSION


def _c_layout(tmp_path, struct, fields):
    src = tmp_path / "layout.c"
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "yl_kvpath.h"', "int main(void) {",
             f'  printf("size %zu\\n", sizeof({struct}));']
    for f in fields:
        lines.append(f'  printf("{f} %zu\\n", offsetof({struct}, {f}));')
    lines += ["  return 0;", "}"]
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{os.path.dirname(HEADER)}", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    return {k: int(v) for k, v in (line.split() for line in out.strip().splitlines())}


@pytest.mark.parametrize("struct,cls", [("yl_store_args", _abi.StoreArgs), ("yl_index_args", _abi.IndexArgs),
                                        ("yl_step_args", _abi.StepArgs), ("yl_gather_args", _abi.GatherArgs),
                                        ("yl_qkv_store_args", _abi.QkvStoreArgs), ("yl_page_pool", _abi.PagePool),
                                        ("yl_reserve_args", _abi.ReserveArgs), ("yl_release_args", _abi.ReleaseArgs),
                                        ("yl_ranges_args", _abi.RangesArgs)])
def test_struct_layout_matches_header(tmp_path, struct, cls):
    names = [f for f, _ in cls._fields_]
    c = _c_layout(tmp_path, struct, names)
    assert c["size"] == ctypes.sizeof(cls)
    for f in names:
        assert c[f] == getattr(cls, f).offset, f


def _store(**kw):
    a = _abi.StoreArgs()
    base = dict(k=0x1000, v=0x2000, k_cache=0x10000, v_cache=0x20000, slots=0x3000, slot_is_int64=1, num_layers=1,
                num_tokens=4, row_bytes=256, k_row_stride=256, v_row_stride=256, cache_row_stride=256)
    base.update(kw)
    for k, v in base.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,status", [
    (dict(num_tokens=-1), _abi.YL_ERR_BAD_SIZE),
    (dict(num_layers=0), _abi.YL_ERR_BAD_SIZE),
    (dict(row_bytes=0), _abi.YL_ERR_BAD_SIZE),
    (dict(k=0), _abi.YL_ERR_NULL_ARG),
    (dict(slots=0), _abi.YL_ERR_NULL_ARG),
    (dict(slot_is_int64=2), _abi.YL_ERR_BAD_SIZE),
    (dict(cache_row_stride=128), _abi.YL_ERR_BAD_SIZE),
    (dict(slots=0x3004), _abi.YL_ERR_ALIGNMENT),
    (dict(num_layers=1 << 20, num_tokens=1 << 12), _abi.YL_ERR_UNSUPPORTED),
])
def test_store_rejects_bad_arguments_on_host(kw, status):
    assert _abi.kv_store_raw(_store(**kw), None) == status
    assert _abi.last_error().startswith("yl_kv_store")


def test_store_zero_tokens_is_noop_without_device():
    # MHAKVCache::StoreKV returns before any launch when N == 0 (mha_kvcache.h:77-79)
    assert _abi.kv_store_raw(_store(num_tokens=0, k=0, v=0, slots=0), None) == _abi.YL_OK
    assert yl.lib().yl_kv_store(None, None) == _abi.YL_ERR_NULL_ARG
    assert yl.lib().yl_build_index(None, None) == _abi.YL_ERR_NULL_ARG


def _index(**kw):
    a = _abi.IndexArgs()
    base = dict(prior_len=0x1000, new_len=0x2000, page_table=0x3000, page_table_stride=8, num_table_rows=4,
                max_pages_per_row=8, page_size=16, batch_size=4, slot_is_int64=1, kv_indptr=0x4000,
                kv_indices=0x5000, kv_last_page_len=0x6000, qo_indptr=0x7000, slot_mapping=0x8000,
                kv_indices_capacity=32, slot_capacity=32)
    base.update(kw)
    for k, v in base.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,status", [
    (dict(batch_size=-1), _abi.YL_ERR_BAD_SIZE),
    (dict(page_size=0), _abi.YL_ERR_BAD_SIZE),
    (dict(kv_indptr=0), _abi.YL_ERR_NULL_ARG),
    (dict(qo_indptr=0), _abi.YL_ERR_NULL_ARG),
    (dict(prior_len=0), _abi.YL_ERR_NULL_ARG),
    (dict(page_table=0), _abi.YL_ERR_NULL_ARG),
    (dict(table_index=0x9000, num_table_rows=0), _abi.YL_ERR_BAD_SIZE),
    (dict(num_table_rows=2), _abi.YL_ERR_BAD_SIZE),
    (dict(kv_indices_capacity=-1), _abi.YL_ERR_BAD_SIZE),
    (dict(slot_mapping=0x8004), _abi.YL_ERR_ALIGNMENT),
    (dict(max_pages_per_row=-1), _abi.YL_ERR_BAD_SIZE),
])
def test_index_rejects_bad_arguments_on_host(kw, status):
    assert _abi.build_index_raw(_index(**kw), None) == status
    assert _abi.last_error().startswith("yl_build_index")


def _gather(**kw):
    a = _abi.GatherArgs()
    base = dict(table=0x10000, out=0x20000, indices=0x3000, index_is_int64=0, num_indices=8, row_bytes=256,
                table_row_stride=256, out_row_stride=256, num_rows=100)
    base.update(kw)
    for k, v in base.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,status", [
    (dict(num_indices=-1), _abi.YL_ERR_BAD_SIZE),
    (dict(row_bytes=0), _abi.YL_ERR_BAD_SIZE),
    (dict(reserved=1), _abi.YL_ERR_BAD_SIZE),
    (dict(index_is_int64=2), _abi.YL_ERR_BAD_SIZE),
    (dict(table=0), _abi.YL_ERR_NULL_ARG),
    (dict(indices=0), _abi.YL_ERR_NULL_ARG),
    (dict(out_row_stride=128), _abi.YL_ERR_BAD_SIZE),
    (dict(indices=0x3002), _abi.YL_ERR_ALIGNMENT),
    (dict(indices=0x3004, index_is_int64=1), _abi.YL_ERR_ALIGNMENT),
    (dict(num_indices=1 << 31), _abi.YL_ERR_UNSUPPORTED),
])
def test_gather_rejects_bad_arguments_on_host(kw, status):
    assert _abi.gather_rows_raw(_gather(**kw), None) == status
    assert _abi.last_error().startswith("yl_gather_rows")


def test_gather_zero_indices_is_noop_without_device():
    assert _abi.gather_rows_raw(_gather(num_indices=0, table=0, out=0, indices=0), None) == _abi.YL_OK
    assert yl.lib().yl_gather_rows(None, None) == _abi.YL_ERR_NULL_ARG


def _qkv(**kw):
    a = _abi.QkvStoreArgs()
    base = dict(q=0x10000, k=0x20000, v=0x30000, q_out=0x40000, k_cache=0x100000, v_cache=0x200000, slots=0x5000,
                dtype=0, slot_is_int64=1, num_q_heads=32, num_kv_heads=8, head_dim=128, eps=1e-6, num_tokens=4,
                q_row_stride=8192, k_row_stride=2048, v_row_stride=2048, q_out_row_stride=8192,
                cache_row_stride=2048, num_slots=1000)
    base.update(kw)
    for k, v in base.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,status", [
    (dict(num_tokens=-1), _abi.YL_ERR_BAD_SIZE),
    (dict(dtype=2), _abi.YL_ERR_BAD_SIZE),
    (dict(head_dim=96), _abi.YL_ERR_UNSUPPORTED),
    (dict(num_kv_heads=0), _abi.YL_ERR_BAD_SIZE),
    (dict(rope_interleaved=2), _abi.YL_ERR_BAD_SIZE),
    (dict(eps=-1.0), _abi.YL_ERR_BAD_SIZE),
    (dict(eps=float("nan")), _abi.YL_ERR_BAD_SIZE),
    (dict(k=0), _abi.YL_ERR_NULL_ARG),
    (dict(q_out=0), _abi.YL_ERR_NULL_ARG),
    (dict(cos_sin_cache=0x9000), _abi.YL_ERR_BAD_SIZE),
    (dict(cos_sin_cache=0x9000, positions=0x6000, max_position=0), _abi.YL_ERR_BAD_SIZE),
    (dict(cache_row_stride=1024), _abi.YL_ERR_BAD_SIZE),
    (dict(q_row_stride=4096), _abi.YL_ERR_BAD_SIZE),
    (dict(k=0x20004), _abi.YL_ERR_ALIGNMENT),
    (dict(k_weight=0x7002), _abi.YL_ERR_ALIGNMENT),
    (dict(cos_sin_cache=0x9008, positions=0x6000, max_position=10), _abi.YL_ERR_ALIGNMENT),
    (dict(slots=0x5004), _abi.YL_ERR_ALIGNMENT),
    (dict(num_tokens=1 << 26), _abi.YL_ERR_UNSUPPORTED),
])
def test_qkv_store_rejects_bad_arguments_on_host(kw, status):
    assert _abi.qkv_store_raw(_qkv(**kw), None) == status
    assert _abi.last_error().startswith("yl_qkv_norm_rope_store")


def test_qkv_store_zero_tokens_is_noop_without_device():
    assert _abi.qkv_store_raw(_qkv(num_tokens=0, q=0, k=0, v=0, slots=0), None) == _abi.YL_OK
    assert yl.lib().yl_qkv_norm_rope_store(None, None) == _abi.YL_ERR_NULL_ARG


def _pool_args(cls, **kw):
    a = cls()
    a.pool = _abi.PagePool(0x1000, 0x2000, 64)
    base = dict(page_table=0x3000, page_table_stride=8, num_table_rows=4, max_pages_per_row=8, page_size=16)
    if cls is _abi.ReserveArgs:
        base.update(prior_len=0x4000, new_len=0x5000, batch_size=4)
    else:
        base.update(rows=0x4000, num_tokens=0x5000, num_release=2)
    for k, v in kw.items():
        if k.startswith("pool_"):
            setattr(a.pool, k[5:], v)
        else:
            base[k] = v
    for k, v in base.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kind", ["reserve", "release"])
@pytest.mark.parametrize("kw,status", [
    (dict(pool_free_pages=0), _abi.YL_ERR_NULL_ARG),
    (dict(pool_capacity=0), _abi.YL_ERR_BAD_SIZE),
    (dict(pool_capacity=1 << 31), _abi.YL_ERR_BAD_SIZE),
    (dict(pool_free_count=0x2002), _abi.YL_ERR_ALIGNMENT),
    (dict(page_table=0), _abi.YL_ERR_NULL_ARG),
    (dict(page_size=0), _abi.YL_ERR_BAD_SIZE),
    (dict(page_table_stride=4), _abi.YL_ERR_BAD_SIZE),
    (dict(page_table=0x3002), _abi.YL_ERR_ALIGNMENT),
])
def test_page_pool_rejects_bad_arguments_on_host(kind, kw, status):
    cls, raw, name = ((_abi.ReserveArgs, _abi.reserve_pages_raw, "yl_reserve_pages") if kind == "reserve" else
                      (_abi.ReleaseArgs, _abi.release_pages_raw, "yl_release_pages"))
    assert raw(_pool_args(cls, **kw), None) == status
    assert _abi.last_error().startswith(name)


def test_page_pool_empty_calls_are_noops_without_device():
    assert _abi.reserve_pages_raw(_pool_args(_abi.ReserveArgs, batch_size=0, pool_free_pages=0), None) == _abi.YL_OK
    assert _abi.release_pages_raw(_pool_args(_abi.ReleaseArgs, num_release=0, page_table=0), None) == _abi.YL_OK
    assert _abi.reserve_pages_raw(_pool_args(_abi.ReserveArgs, batch_size=-1), None) == _abi.YL_ERR_BAD_SIZE
    assert _abi.reserve_pages_raw(_pool_args(_abi.ReserveArgs, batch_size=5), None) == _abi.YL_ERR_BAD_SIZE
    assert _abi.reserve_pages_raw(_pool_args(_abi.ReserveArgs, new_len=0), None) == _abi.YL_ERR_NULL_ARG
    assert yl.lib().yl_reserve_pages(None, None) == _abi.YL_ERR_NULL_ARG
    assert yl.lib().yl_release_pages(None, None) == _abi.YL_ERR_NULL_ARG


def _ranges(**kw):
    a = _abi.RangesArgs()
    base = dict(ranges=0x10000, indices=0x20000, count=0x30000, num_ranges=4, indices_capacity=100, error_word=0x40000)
    base.update(kw)
    for k, v in base.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,status", [
    (dict(num_ranges=-1), _abi.YL_ERR_BAD_SIZE),
    (dict(indices_capacity=-1), _abi.YL_ERR_BAD_SIZE),
    (dict(num_ranges=(1 << 22) + 1), _abi.YL_ERR_UNSUPPORTED),
    (dict(indices_capacity=1 << 40), _abi.YL_ERR_UNSUPPORTED),
    (dict(ranges=0), _abi.YL_ERR_NULL_ARG),
    (dict(indices=0), _abi.YL_ERR_NULL_ARG),
    (dict(ranges=0x10004), _abi.YL_ERR_ALIGNMENT),
    (dict(indices=0x20002), _abi.YL_ERR_ALIGNMENT),
    (dict(count=0x30001), _abi.YL_ERR_ALIGNMENT),
])
def test_make_2d_indices_rejects_bad_arguments_on_host(kw, status):
    assert _abi.make_2d_indices_raw(_ranges(**kw), None) == status
    assert _abi.last_error().startswith("yl_make_2d_indices")


def test_make_2d_indices_empty_call_is_noop_without_device():
    assert _abi.make_2d_indices_raw(_ranges(num_ranges=0, count=0, ranges=0, indices=0), None) == _abi.YL_OK
    assert yl.lib().yl_make_2d_indices(None, None) == _abi.YL_ERR_NULL_ARG


def _header_defines(prefix):
    text = open(HEADER).read()
    return {m.group(1): int(m.group(2), 16) for m in re.finditer(rf"#define ({prefix}\w+)\s+(0x[0-9a-fA-F]+)u?", text)}


def test_error_bits_and_statuses_agree_with_header():
    """Every device error bit of the header has the same value in the Python
    binding, and the oracle's bits are the header's; status codes likewise."""
    from oracle import kvpath as orc

    bits = _header_defines("YL_DEVERR_")
    assert len(bits) >= 14 and len(set(bits.values())) == len(bits)
    for name, value in bits.items():
        short = name[len("YL_DEVERR_"):]
        assert getattr(_abi, "DEVERR_" + short) == value, name
        if hasattr(orc, short):
            assert getattr(orc, short) == value, name
    text = open(HEADER).read()
    for m in re.finditer(r"(YL_(?:OK|ERR_\w+))\s*=\s*(-?\d+)", text):
        assert getattr(_abi, m.group(1)) == int(m.group(2)), m.group(1)
        assert _abi.status_string(int(m.group(2))) == m.group(1)


def test_status_strings():
    assert _abi.status_string(0) == "YL_OK"
    assert _abi.status_string(-3) == "YL_ERR_ALIGNMENT"
    with pytest.raises(yl.KVPathError, match="YL_ERR_BAD_SIZE"):
        _abi.check(_abi.kv_store_raw(_store(num_tokens=-1), None))


def test_launch_without_device_reports_cuda_error():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a device is present")
    # valid arguments, no GPU: the launch must fail with a status, not crash
    assert _abi.kv_store_raw(_store(), None) == _abi.YL_ERR_CUDA


FASTDIV_PROBE = r"""
#include <cstdio>
#include <cstdint>
#include "common.cuh"
int main() {
  const uint32_t divs[] = {1, 2, 3, 5, 7, 16, 17, 64, 100, 255, 256, 257, 1000, 4096, 65535, 65536, 65537,
                           1000003, 123456789, 1u << 30, (1u << 30) + 1, 2147483647u};
  const uint32_t nums[] = {0, 1, 2, 3, 15, 16, 17, 255, 256, 65535, 65536, 999999, 1u << 20, 123456789,
                           1u << 30, (1u << 30) + 7, 2147483646u, 2147483647u};
  long bad = 0;
  for (uint32_t d : divs) {
    ylk::FastDiv f(d);
    for (uint32_t n : nums) if (f.div(n) != n / d) ++bad;
    for (uint32_t n = 0; n < 200000; ++n) if (f.div(n) != n / d) ++bad;
    for (uint32_t q = 1; q < 4096; ++q) {               // around multiples of d
      const uint64_t m = (uint64_t)q * d;
      for (int dd = -1; dd <= 1; ++dd) {
        const uint64_t n = m + dd;
        if (n < (1ull << 31) && f.div((uint32_t)n) != (uint32_t)n / d) ++bad;
      }
    }
  }
  printf("%ld\n", bad);
  return 0;
}
"""


def test_fastdiv_exact(tmp_path):
    src = tmp_path / "fastdiv.cu"
    src.write_text(FASTDIV_PROBE)
    exe = tmp_path / "fastdiv"
    csrc = os.path.join(ROOT, "yllang_b200", "csrc")
    subprocess.run(["nvcc", "-std=c++17", "-O2", f"-I{csrc}", f"-I{os.path.dirname(HEADER)}", str(src), "-o",
                    str(exe)], check=True)
    assert subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.strip() == "0"


def test_missing_library_fails_loudly(tmp_path):
    """Without libyl_kvpath.so the package raises instead of falling back to
    any host path (run in a child so this process keeps its library)."""
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "from yllang_b200 import _abi\n"
        "_abi.LIB_PATH = %r\n"
        "_abi._lib = None\n"
        "try:\n"
        "    _abi.lib()\n"
        "except ImportError as e:\n"
        "    print('refused:', e)\n"
        "else:\n"
        "    print('loaded')\n" % (ROOT, str(tmp_path / "libyl_kvpath.so"))
    )
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.startswith("refused:") and "build the CUDA library" in r.stdout


def test_python_ops_refuse_host_tensors_and_bad_shapes():
    """The Python front end's checks run before any launch: host tensors,
    wrong dtypes and shapes raise PanicError (no CPU path exists)."""
    import torch

    with pytest.raises(yl.PanicError, match="CUDA"):
        yl.make_2d_indices(torch.zeros(2, 3, dtype=torch.int64))
    with pytest.raises(yl.PanicError, match="CUDA"):
        yl.gather_rows(torch.zeros(3, dtype=torch.int32), torch.zeros(10, 64))
    with pytest.raises(yl.PanicError, match="CUDA"):
        yl.store_kv_cache(*(torch.zeros(4, 64) for _ in range(2)), *(torch.zeros(16, 64) for _ in range(2)),
                          torch.zeros(4, dtype=torch.int64))


def test_device_error_names_and_debug_mode_default_off():
    C = yl.load_extension()
    for bits, want in [(0, ""), (0x1, "SLOT_RANGE"), (0x401, "SLOT_RANGE|INDEX_RANGE"),
                       (0x3000, "POOL_EMPTY|POOL_OVERFLOW"), (0x10002, "PAGE_RANGE|0x10000"), (0x40000, "0x40000")]:
        assert _abi.deverr_names(bits) == want
        assert C.DeviceErrorNames(bits) == want
    if not os.environ.get("YLLANG_CHECK_DEVICE_ERRORS"):
        assert not yl.ops.CHECK_DEVICE_ERRORS and not C.DeviceErrorChecksEnabled()


def test_attention_library_exports_every_declared_symbol():
    """include/yl_attention.h declares the C entry points of
    libyl_attention.so; the library exports exactly those (its C++ bridge
    functions are exported C++ symbols, not yl_*)."""
    text = open(os.path.join(ROOT, "include", "yl_attention.h")).read()
    declared = sorted(set(re.findall(r"YL_API\s+[\w\s\*]*?\b(yl_\w+)\s*\(", text)))
    lib = os.path.join(ROOT, "yllang_b200", "libyl_attention.so")
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True)
    assert sorted(set(re.findall(r" T (yl_\w+)", out.stdout))) == declared
    f = ctypes.CDLL(lib).yl_paged_decode_attention_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    assert f(None, None) == -1  # YL_ERR_NULL_ARG, checked on the host before any launch
