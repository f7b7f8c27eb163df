"""KV store on the GPU vs the CPU oracle, through the C ABI (bit-exact).

Pools are filled with random sentinel bytes first, so a stray write anywhere
in the pool shows up as a mismatch against the oracle's copy of the pool.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import yllang_b200 as yl
from _kvutil import host_bytes, oracle_store, random_bytes
from yllang_b200 import workloads

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _case(dev, N, S, row_bytes, L=1, slot_dtype=torch.int64, seed=0, pad=0, in_stride_extra=0):
    """Random inputs and a sentinel-filled pool as uint8 rows."""
    g = torch.Generator().manual_seed(seed)
    shape_in = (L, N, row_bytes + in_stride_extra) if L > 1 else (N, row_bytes + in_stride_extra)
    kbuf = random_bytes(shape_in, seed + 1).to(dev)
    vbuf = random_bytes(shape_in, seed + 2).to(dev)
    k = kbuf[..., :row_bytes]
    v = vbuf[..., :row_bytes]
    pool_shape = (L, S, row_bytes) if L > 1 else (S, row_bytes)
    k_cache = random_bytes(pool_shape, seed + 3).to(dev)
    v_cache = random_bytes(pool_shape, seed + 4).to(dev)
    slots = torch.randperm(S, generator=g)[:N]
    if pad:
        slots[torch.randperm(N, generator=g)[:pad]] = -1
    return k, v, k_cache, v_cache, slots.to(slot_dtype).to(dev)


def _check(k, v, k_cache, v_cache, slots, num_slots=0):
    want_k, want_v, want_err = oracle_store(k, v, k_cache, v_cache, slots, num_slots)
    err = torch.zeros(1, dtype=torch.int32, device=k.device)
    yl.store_kv_cache(k, v, k_cache, v_cache, slots, error_word=err)
    torch.cuda.synchronize()
    assert np.array_equal(host_bytes(k_cache), want_k)
    assert np.array_equal(host_bytes(v_cache), want_v)
    assert int(err.item()) == want_err


ROW_BYTES = [16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 48, 96, 192, 1536, 3072, 24, 12, 6, 2, 1]


@pytest.mark.parametrize("row_bytes", ROW_BYTES)
@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64])
def test_store_row_sizes(cuda, row_bytes, slot_dtype):
    _check(*_case(cuda, N=173, S=600, row_bytes=row_bytes, slot_dtype=slot_dtype, seed=row_bytes, pad=5))


@pytest.mark.parametrize("row_bytes", [256, 1024, 2048, 4096])
@pytest.mark.parametrize("L", [2, 5])
def test_store_all_layers_one_launch(cuda, row_bytes, L):
    _check(*_case(cuda, N=257, S=1000, row_bytes=row_bytes, L=L, seed=L * 7 + row_bytes))


@pytest.mark.parametrize("extra", [16, 48, 1024])
def test_store_strided_inputs(cuda, extra):
    # rows taken out of a wider buffer (e.g. the K part of a packed QKV row)
    _check(*_case(cuda, N=99, S=300, row_bytes=2048, seed=extra, in_stride_extra=extra))
    _check(*_case(cuda, N=99, S=300, row_bytes=1024, L=3, seed=extra + 1, in_stride_extra=extra))


def test_store_misaligned_inputs_take_generic_path(cuda):
    # 8-byte aligned row starts: still exact
    _check(*_case(cuda, N=64, S=200, row_bytes=2048, seed=5, in_stride_extra=8))


def test_store_bf16_pool_view(cuda):
    # bf16 K/V [N, H, D] into the per-layer [P * ps, H * D] view of a [2, L, P, ps, H, D] pool
    torch.manual_seed(0)
    L, P, ps, H, D, N = 3, 64, 16, 8, 128, 200
    pool = torch.randn(2, L, P, ps, H, D).to(torch.bfloat16).to(cuda)
    k = torch.randn(N, H, D).to(torch.bfloat16).to(cuda)
    v = torch.randn(N, H, D).to(torch.bfloat16).to(cuda)
    slots = torch.randperm(P * ps)[:N].to(cuda)
    layer = 1
    kc = pool[0, layer].view(P * ps, H * D)
    vc = pool[1, layer].view(P * ps, H * D)
    before = pool.clone()
    _check(k.view(N, -1), v.view(N, -1), kc, vc, slots, num_slots=P * ps)
    # other layers untouched
    others = [l for l in range(L) if l != layer]
    assert torch.equal(pool[:, others].view(torch.int16), before[:, others].view(torch.int16))


def test_store_out_of_range_slots_reported(cuda):
    k, v, kc, vc, slots = _case(cuda, N=50, S=100, row_bytes=512, seed=11)
    slots[3] = 100  # == num_slots
    slots[7] = -5
    slots[9] = -1  # padding: silent
    _check(k, v, kc, vc, slots, num_slots=100)


def test_store_later_call_wins(cuda):
    # TestStoreKVOverwritesSamePage / TestStoreKVMultipleRandomWrites, seeded
    S, E = 128, 512
    g = torch.Generator().manual_seed(3)
    kc = torch.zeros(S, E, dtype=torch.uint8, device=cuda)
    vc = torch.zeros_like(kc)
    kc_ref = np.zeros((S, E), np.uint8)
    vc_ref = np.zeros_like(kc_ref)
    from oracle import kvpath as orc
    for it in range(300):
        n = int(torch.randint(1, 13, (1,), generator=g))
        slots = torch.randperm(S, generator=g)[:n]
        k = random_bytes((n, E), 1000 + it)
        v = random_bytes((n, E), 5000 + it)
        yl.store_kv_cache(k.to(cuda), v.to(cuda), kc, vc, slots.to(cuda))
        orc.store(k.numpy(), v.numpy(), kc_ref, vc_ref, slots.numpy())
    torch.cuda.synchronize()
    assert np.array_equal(kc.cpu().numpy(), kc_ref) and np.array_equal(vc.cpu().numpy(), vc_ref)


def test_store_empty_is_noop(cuda):
    kc = torch.ones(8, 512, dtype=torch.uint8, device=cuda)
    e = torch.empty(0, 512, dtype=torch.uint8, device=cuda)
    yl.store_kv_cache(e, e, kc, kc.clone(), torch.empty(0, dtype=torch.int64, device=cuda))
    torch.cuda.synchronize()
    assert (kc == 1).all()


def test_store_rejects_contract_violations(cuda):
    k = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda)
    kc = torch.zeros(16, 64, dtype=torch.bfloat16, device=cuda)
    s = torch.arange(4, device=cuda)
    with pytest.raises(yl.PanicError):
        yl.store_kv_cache(k, k, kc, kc.float(), s)  # dtype mismatch
    with pytest.raises(yl.PanicError):
        yl.store_kv_cache(k, k, kc[:, :32], kc[:, :32], s)  # row size mismatch
    with pytest.raises(yl.PanicError):
        yl.store_kv_cache(k, k, kc, kc, s[:3])  # slot count
    with pytest.raises(yl.PanicError):
        yl.store_kv_cache(k, k, kc, kc, s.float())  # slot dtype


@pytest.mark.parametrize("make", ["cpu_ref", "llama3_decode", "mixed"])
def test_store_workload_slots(cuda, make):
    """Store with the slot mapping of a workload's batch (bf16, per-layer and all-layer forms)."""
    if make == "cpu_ref":
        b = workloads.cpu_ref()
    elif make == "llama3_decode":
        b = workloads.llama3_decode(num_pages=70000, layers=2)
    else:
        b = workloads.mixed(num_pages=4000, page_size=16, head_dim=256, layers=2)
    from oracle import kvpath as orc
    ref = orc.build_index(b.prior_len, b.new_len, b.page_table, b.page_size, num_pages=b.num_pages)
    slots = torch.from_numpy(ref["slot_mapping"]).to(cuda)
    S = b.num_pages * b.page_size
    E = b.kv_heads * b.head_dim
    torch.manual_seed(0)
    L = b.layers
    k = torch.randn(L, b.tokens, E).to(torch.bfloat16).to(cuda)
    v = torch.randn(L, b.tokens, E).to(torch.bfloat16).to(cuda)
    kc = torch.zeros(L, S, E, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    yl.store_kv_cache(k, v, kc, vc, slots, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # check every written row and a checksum of the whole pool
    s = slots.long()
    assert torch.equal(kc[:, s].view(torch.int16), k.view(torch.int16))
    assert torch.equal(vc[:, s].view(torch.int16), v.view(torch.int16))
    written = torch.zeros(S, dtype=torch.bool, device=cuda)
    written[s] = True
    assert int(kc[:, ~written].view(torch.int16).abs().sum()) == 0


def test_store_vector16_variant_matches(cuda):
    """The 16-byte-vector fast path (YL_STORE_VECTOR_BYTES=16) is bit-exact too."""
    code = (
        "import sys; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
        "import torch, numpy as np, yllang_b200 as yl\n"
        "from _kvutil import random_bytes, oracle_store, host_bytes\n"
        "dev = torch.device('cuda:0')\n"
        "for rb in (256, 512, 1024, 2048, 4096, 8192):\n"
        "  for L in (1, 3):\n"
        "    sh = (L, 300, rb) if L > 1 else (300, rb)\n"
        "    ps = (L, 900, rb) if L > 1 else (900, rb)\n"
        "    k = random_bytes(sh, rb).to(dev); v = random_bytes(sh, rb + 1).to(dev)\n"
        "    kc = random_bytes(ps, rb + 2).to(dev); vc = random_bytes(ps, rb + 3).to(dev)\n"
        "    s = torch.randperm(900)[:300].to(dev)\n"
        "    wk, wv, _ = oracle_store(k, v, kc, vc, s)\n"
        "    yl.store_kv_cache(k, v, kc, vc, s); torch.cuda.synchronize()\n"
        "    assert np.array_equal(host_bytes(kc), wk) and np.array_equal(host_bytes(vc), wv), (rb, L)\n"
        "print('ok')\n" % (ROOT, os.path.join(ROOT, "tests")))
    env = dict(os.environ, YL_STORE_VECTOR_BYTES="16")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]


@pytest.mark.parametrize("env", [{"YL_STORE_ENGINE": "tma"}, {"YL_STORE_ENGINE": "tma", "YL_STEP_MODE": "serial"}])
def test_store_engines_match(cuda, env):
    """The TMA-staged store engine passes the store and step suites too (the
    engine is read once per process, so run them in a child)."""
    here = os.path.dirname(os.path.abspath(__file__))
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(here, "test_store_gpu.py"), os.path.join(here, "test_step_gpu.py"),
                        os.path.join(here, "test_ref_kernel_gpu.py"),
                        "-k", "not engines_match and not other_modes and not vector16"],
                       env=dict(os.environ, **env), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
