"""Debug mode (YLLANG_CHECK_DEVICE_ERRORS=1): calls given no device error
word read the kernels' error bits back and raise PanicError naming them, in
the Python and the C++ front ends; valid calls pass.  The bad inputs are the
ones the kernels skip and flag (a slot past the pool, an embedding id past the
table, a page id past the pool, more pages than the pool holds), never an
access outside a buffer.  Runs in a child process, since the mode is read once
per process.  Also: an error word that is not a 4-byte tensor on the call's
device is refused before any launch."""
import os
import subprocess
import sys

import pytest
import torch

import yllang_b200 as yl

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import torch
import yllang_b200 as yl

C = yl.load_extension()
assert yl.ops.CHECK_DEVICE_ERRORS and C.DeviceErrorChecksEnabled()
dev = torch.device("cuda:0")


def raises(fn, name, exc):
    try:
        fn()
    except exc as e:
        assert name in str(e), str(e)
        return
    raise SystemExit(f"no error raised for {name}")


g = torch.Generator(device=dev).manual_seed(1)
k = torch.randn(4, 256, device=dev, generator=g).to(torch.bfloat16)
v = torch.randn(4, 256, device=dev, generator=g).to(torch.bfloat16)
kc = torch.zeros(64, 256, dtype=torch.bfloat16, device=dev)
vc = torch.zeros_like(kc)
ok = torch.tensor([0, 1, 2, 3], device=dev)
bad = torch.tensor([0, 1, 64, 3], device=dev)
yl.store_kv_cache(k, v, kc, vc, ok)
raises(lambda: yl.store_kv_cache(k, v, kc, vc, bad), "SLOT_RANGE", yl.PanicError)
C.StoreKVCache(k, v, kc, vc, ok + 4)
raises(lambda: C.StoreKVCache(k, v, kc, vc, bad), "SLOT_RANGE", C.PanicError)
assert torch.equal(kc[:8], torch.cat([k, k])) and torch.equal(vc[:8], torch.cat([v, v]))

w = torch.randn(10, 64, device=dev, generator=g)
yl.gather_rows(torch.tensor([1, 9], device=dev), w)
raises(lambda: yl.gather_rows(torch.tensor([1, 10], device=dev), w), "INDEX_RANGE", yl.PanicError)
raises(lambda: C.Index(torch.tensor([12, 0], device=dev), w, torch.empty(2, 64, device=dev)), "INDEX_RANGE",
       C.PanicError)

i32 = dict(dtype=torch.int32, device=dev)
table = torch.tensor([[0, 1], [2, 50]], **i32)
prior, new = torch.tensor([3, 20], **i32), torch.tensor([1, 1], **i32)
yl.build_index(prior, new, table, 16, num_pages=64)
raises(lambda: yl.build_index(prior, new, table, 16, num_pages=40), "PAGE_RANGE", yl.PanicError)
raises(lambda: C.BuildBatchIndex(prior, new, table, 16, num_pages=40), "PAGE_RANGE", C.PanicError)

pool = yl.DevicePagePool(4, dev)
pt = torch.full((2, 8), -1, **i32)
raises(lambda: pool.reserve(pt, torch.zeros(2, **i32), torch.tensor([64, 64], **i32), 16), "POOL_EMPTY",
       yl.PanicError)
assert pool.free_count() == 4 and bool((pt == -1).all())
cpool = C.DevicePagePool(4, "cuda:0")
raises(lambda: cpool.Reserve(pt, torch.zeros(2, **i32), torch.tensor([64, 64], **i32), 16), "POOL_EMPTY",
       C.PanicError)

# calls on a side stream: the private word is zeroed on that stream and read
# after it finishes, so a kernel queued behind a long one is still checked
side = torch.cuda.Stream(dev)
big = torch.empty(1 << 28, dtype=torch.uint8, device=dev)
side.wait_stream(torch.cuda.current_stream(dev))
for _ in range(3):
    with torch.cuda.stream(side):
        big.random_(0, 255)  # keeps the side stream busy past the current stream's work
    raises(lambda: yl.store_kv_cache(k, v, kc, vc, bad, stream=side), "SLOT_RANGE", yl.PanicError)
    raises(lambda: yl.gather_rows(torch.tensor([1, 10], device=dev), w, stream=side), "INDEX_RANGE",
           yl.PanicError)
    yl.store_kv_cache(k, v, kc, vc, ok, stream=side)
with torch.cuda.stream(side):
    rng = torch.tensor([[0, 0, 3], [100, 2, 4]], dtype=torch.int64, device=dev)
flat = yl.make_2d_indices(rng, stream=side)
assert flat.tolist() == [0, 1, 2, 102, 103]
torch.cuda.synchronize()
print("device error checks ok")
"""


def test_debug_mode_raises_on_device_error_bits(cuda):
    env = dict(os.environ, YLLANG_CHECK_DEVICE_ERRORS="1")
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "device error checks ok" in r.stdout


def test_error_word_must_live_on_the_call_device(cuda):
    C = yl.load_extension()
    w = torch.randn(10, 64, device=cuda)
    idx = torch.tensor([1, 2], device=cuda)
    for word in (torch.zeros(1, dtype=torch.int32), torch.zeros(1, dtype=torch.int64, device=cuda)):
        with pytest.raises(yl.PanicError, match="error_word"):
            yl.gather_rows(idx, w, error_word=word)
    i32 = dict(dtype=torch.int32, device=cuda)
    pool = C.DevicePagePool(4, "cuda:0")
    with pytest.raises(C.PanicError, match="error_word"):
        pool.Reserve(torch.full((1, 2), -1, **i32), torch.zeros(1, **i32), torch.ones(1, **i32), 16,
                     error_word=torch.zeros(1, dtype=torch.int32))
    with pytest.raises(C.PanicError, match="error_word"):
        C.BuildBatchIndex(torch.zeros(1, **i32), torch.ones(1, **i32), torch.zeros(1, 2, **i32), 16,
                          error_word=torch.zeros(1, dtype=torch.int32))
