"""Bit-exact parity at the full sizes of the five workloads the benchmark
runs, through the same public step the benchmark times (yllang_b200.kv_step)
and through the two separate calls:

* Llama-3-8B decode: 256 sequences, 32 layers, 2 KB rows; and the per-rank
  shapes of its head-sharded runs (512 / 1,024 / 2,048 sequences at 4 / 2 / 1
  KV heads, 1,024- to 256-byte rows);
* ragged prefill: 64 prompts U[128, 4096] (~131 k tokens), 32 layers;
* Qwen2-72B decode: 512 sequences, 80 layers, at 8 / 4 / 2 / 1 KV heads per
  GPU (2,048- to 256-byte rows);
* the mixed batch (128 decode + 8 prefill chunks of 512), 4 layers, at every
  (page size, head dim) pair of {1, 16, 64} x {64, 128, 256}.

Every element of the five index arrays is compared with the C oracle; the
pool is filled with random sentinel bytes first and kept as a copy, every
written row is compared with its input row, and after the written rows are
put back from the copy the whole pool must equal the copy, so a stray write
anywhere shows.  Pools are smaller than the benchmark's 150 GB: pages that are
only read alias other pool pages, the pages written in the step stay unique,
which changes no kernel path (grids depend on the batch, rows and layers)."""
import numpy as np
import pytest
import torch

import yllang_b200 as yl
from _kvutil import assert_index_equal, index_outputs
from oracle import kvpath as orc
from yllang_b200 import workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _release_device_memory():
    """Hand the tens of GB these tests cache back to the device, so tests that
    run a child process afterwards can allocate."""
    yield
    import gc
    gc.collect()
    torch.cuda.empty_cache()


def _dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)


def _full_step(dev, b, path="step", seed=0):
    L, E = b.layers, b.kv_heads * b.head_dim
    S = b.num_pages * b.page_size
    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.randn(L, b.tokens, E, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(L, b.tokens, E, generator=g, device=dev).to(torch.bfloat16)
    pool = torch.empty(2, L, S, E, dtype=torch.bfloat16, device=dev)
    pool.view(torch.int16).random_(-2**15, 2**15, generator=g)  # sentinel bytes
    orig = pool.clone()
    want = orc.build_index(b.prior_len, b.new_len, b.page_table, b.page_size, num_pages=b.num_pages)
    assert want["err"] == 0
    i32 = dict(dtype=torch.int32, device=dev)
    out = yl.BatchIndex(torch.empty(b.batch + 1, **i32), torch.empty(b.total_pages, **i32),
                        torch.empty(b.batch, **i32), torch.empty(b.batch + 1, **i32),
                        torch.empty(b.tokens, dtype=torch.int64, device=dev))
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    prior, new, table = _dev(b.prior_len, dev), _dev(b.new_len, dev), _dev(b.page_table, dev)
    if path == "step":
        yl.kv_step(prior, new, table, b.page_size, k, v, pool[0], pool[1], out, num_pages=b.num_pages, error_word=err)
    else:
        yl.build_index(prior, new, table, b.page_size, num_pages=b.num_pages, out=out, error_word=err)
        yl.store_kv_cache(k, v, pool[0], pool[1], out.slot_mapping, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert_index_equal(index_outputs(out), want)
    slots = torch.from_numpy(want["slot_mapping"]).to(dev)
    assert torch.unique(slots).numel() == b.tokens  # the step's slots are distinct
    for layer in range(L):
        assert torch.equal(pool[0, layer].index_select(0, slots), k[layer]), f"K rows of layer {layer}"
        assert torch.equal(pool[1, layer].index_select(0, slots), v[layer]), f"V rows of layer {layer}"
        pool[0, layer].index_copy_(0, slots, orig[0, layer].index_select(0, slots))
        pool[1, layer].index_copy_(0, slots, orig[1, layer].index_select(0, slots))
    assert torch.equal(pool.view(torch.int16), orig.view(torch.int16)), "a row outside the step's slots changed"


@pytest.mark.parametrize("path", ["step", "calls"])
def test_llama3_decode_full(cuda, path):
    _full_step(cuda, workloads.llama3_decode(num_pages=8192), path)


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_llama3_decode_rank_shapes(cuda, ranks):
    """Each rank of a G-GPU run: 256 G sequences, 8 / G heads, 32 layers."""
    _full_step(cuda, workloads.llama3_decode(num_pages=12000, batch=256 * ranks, kv_heads=8 // ranks), seed=ranks)


def test_ragged_prefill_full(cuda):
    b = workloads.ragged_prefill(num_pages=8600)
    assert b.batch == 64 and b.tokens > 120_000
    _full_step(cuda, b)


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_qwen72b_decode_full(cuda, tp):
    _full_step(cuda, workloads.qwen72b_decode(num_pages=2048, tp=tp), seed=tp)


@pytest.mark.parametrize("ps", [1, 16, 64])
@pytest.mark.parametrize("hd", [64, 128, 256])
def test_mixed_full(cuda, ps, hd):
    _full_step(cuda, workloads.mixed(num_pages={1: 600_000, 16: 40_000, 64: 10_000}[ps], page_size=ps, head_dim=hd),
               seed=ps + hd)
