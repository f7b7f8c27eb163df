"""The step (yl_kv_step: index build + store of every layer, two overlapped
launches) vs the separate entry points and the CPU oracle (bit-exact)."""
import numpy as np
import pytest
import torch

import yllang_b200 as yl
from _kvutil import assert_index_equal, host_bytes, index_outputs, random_bytes
from oracle import kvpath as orc
from yllang_b200 import workloads

pytestmark = pytest.mark.gpu


def _dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)


def _outs(b, dev, slot_dtype=torch.int64, extra_slots=0):
    i32 = dict(dtype=torch.int32, device=dev)
    return yl.BatchIndex(torch.empty(b.batch + 1, **i32), torch.empty(b.total_pages, **i32),
                         torch.empty(b.batch, **i32), torch.empty(b.batch + 1, **i32),
                         torch.empty(b.tokens + extra_slots, dtype=slot_dtype, device=dev))


def _step_vs_oracle(dev, b, layers_form=True, slot_dtype=torch.int64, table_index=None, seed=0, extra_slots=0,
                    elem=torch.bfloat16):
    S = b.num_pages * b.page_size
    E = b.kv_heads * b.head_dim
    L = b.layers
    g = torch.Generator(device=dev).manual_seed(seed)
    shape = (L, b.tokens, E) if layers_form else (b.tokens, E)
    k = torch.randn(shape, generator=g, device=dev).to(elem)
    v = torch.randn(shape, generator=g, device=dev).to(elem)
    pshape = (L, S, E) if layers_form else (S, E)
    kc = torch.randn(pshape, generator=g, device=dev).to(elem)
    vc = torch.randn(pshape, generator=g, device=dev).to(elem)
    table = b.page_table
    tix_np = None
    if table_index is not None:  # scatter the rows over a bigger table
        R = b.batch + 9
        big = np.full((R, table.shape[1]), -1, np.int32)
        tix_np = np.random.default_rng(seed).permutation(R)[: b.batch].astype(np.int32)
        big[tix_np] = table
        table = big
    want = orc.build_index(b.prior_len, b.new_len, table, b.page_size, table_index=tix_np, num_pages=b.num_pages,
                           slot_dtype=np.int64 if slot_dtype == torch.int64 else np.int32,
                           slot_capacity=b.tokens + extra_slots)
    want_k, want_v = host_bytes(kc).copy(), host_bytes(vc).copy()
    orc.store(host_bytes(k), host_bytes(v), want_k, want_v, want["slot_mapping"][: b.tokens], num_slots=S)
    out = _outs(b, dev, slot_dtype, extra_slots)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    yl.kv_step(_dev(b.prior_len, dev), _dev(b.new_len, dev), _dev(table, dev), b.page_size, k, v, kc, vc, out,
               table_index=None if tix_np is None else _dev(tix_np, dev), num_pages=b.num_pages, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == want["err"] == 0
    got = index_outputs(out)
    assert_index_equal(got, want)
    assert np.array_equal(got["slot_mapping"], want["slot_mapping"])  # including the -1 tail
    assert torch.equal(kc.view(torch.uint8).view(-1), torch.from_numpy(want_k.reshape(-1)).to(dev))
    assert torch.equal(vc.view(torch.uint8).view(-1), torch.from_numpy(want_v.reshape(-1)).to(dev))


def test_step_cpu_ref(cuda):
    _step_vs_oracle(cuda, workloads.cpu_ref(), layers_form=False)


@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64])
def test_step_llama3_decode_shape(cuda, slot_dtype):
    b = workloads.llama3_decode(num_pages=4096, layers=3)  # read-only pages alias, written ones unique
    _step_vs_oracle(cuda, b, slot_dtype=slot_dtype)


@pytest.mark.parametrize("ps", [1, 16, 64])
@pytest.mark.parametrize("hd", [64, 128, 256])
def test_step_mixed(cuda, ps, hd):
    b = workloads.mixed(num_pages=20000 if ps == 1 else 6000, page_size=ps, head_dim=hd, layers=2)
    _step_vs_oracle(cuda, b, table_index=True, seed=ps + hd)


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_step_head_shards(cuda, tp):
    b = workloads.qwen72b_decode(num_pages=20000, tp=tp, batch=128, layers=3, ctx_hi=8192)
    _step_vs_oracle(cuda, b)


def test_step_prefill_chunks(cuda):
    b = workloads.ragged_prefill(num_pages=12000, requests=12, layers=2, hi=2048)
    _step_vs_oracle(cuda, b)


def test_step_slot_tail_and_fp32(cuda):
    b = workloads.cpu_ref()
    _step_vs_oracle(cuda, b, layers_form=False, extra_slots=37, elem=torch.float32)


def test_step_large_batch_falls_back(cuda):
    # more than 4096 sequences: index build and store run as two launches
    b = workloads.llama3_decode(num_pages=8000, batch=5000, layers=1, ctx_lo=16, ctx_hi=64)
    _step_vs_oracle(cuda, b)


def test_step_generic_rows_fall_back(cuda):
    # 24-byte rows have no 16-byte fast shape: two launches, same result
    rng = np.random.default_rng(3)
    prior = rng.integers(0, 40, 20).astype(np.int32)
    new = rng.integers(0, 5, 20).astype(np.int32)
    ps, P = 4, 400
    pps = (prior.astype(np.int64) + new + ps - 1) // ps
    table = workloads._page_table(pps, new, prior, ps, P, np.random.default_rng(4))
    b = workloads.Batch("odd", 2, 1, 12, ps, P, prior, new, table)
    _step_vs_oracle(cuda, b)


def test_step_token_count_mismatch_flags(cuda):
    b = workloads.cpu_ref()
    out = _outs(b, cuda, extra_slots=4)
    E = b.kv_heads * b.head_dim
    N = b.tokens + 4  # four rows more than the lengths account for
    k = torch.randn(N, E, device=cuda).to(torch.bfloat16)
    kc = torch.zeros(b.num_pages * b.page_size, E, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    yl.kv_step(_dev(b.prior_len, cuda), _dev(b.new_len, cuda), _dev(b.page_table, cuda), b.page_size, k, k, kc, vc,
               out, num_pages=b.num_pages, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) & yl.DEVERR_TOKEN_COUNT
    s = out.slot_mapping.cpu().numpy()
    assert (s[b.tokens:] == -1).all() and (s[: b.tokens] >= 0).all()
    # the extra rows were not stored anywhere: exactly the batch's rows are non-zero
    assert int((kc.view(torch.int16) != 0).any(dim=1).sum()) == b.tokens


def test_step_bad_page_skips_rows(cuda):
    b = workloads.cpu_ref()
    b.page_table = b.page_table.copy()
    b.page_table[4, 1] = b.num_pages + 5  # a page of the prefill request outside the pool
    out = _outs(b, cuda)
    E = b.kv_heads * b.head_dim
    k = torch.randn(b.tokens, E, device=cuda).to(torch.bfloat16)
    kc = torch.zeros(b.num_pages * b.page_size, E, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    yl.kv_step(_dev(b.prior_len, cuda), _dev(b.new_len, cuda), _dev(b.page_table, cuda), b.page_size, k, k, kc, vc,
               out, num_pages=b.num_pages, error_word=err)
    torch.cuda.synchronize()
    want = orc.build_index(b.prior_len, b.new_len, b.page_table, b.page_size, num_pages=b.num_pages)
    assert int(err.item()) == want["err"] and want["err"] & orc.PAGE_RANGE
    assert np.array_equal(out.slot_mapping.cpu().numpy(), want["slot_mapping"])
    assert int((kc.view(torch.int16) != 0).any(dim=1).sum()) == int((want["slot_mapping"] >= 0).sum())


@pytest.mark.parametrize("mode", ["serial"])
def test_step_other_modes(cuda, mode):
    """The serial two-launch form (the store waits for the whole index build
    and reads its slots) gives the same results as the default overlapped
    form (the mode is read once per process, so run in a child)."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, YL_STEP_MODE=mode)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(here, "test_step_gpu.py"), "-k", "not other_modes"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.parametrize("B", [200, 300, 1500])
@pytest.mark.parametrize("tix,slot_dtype", [(False, torch.int64), (True, torch.int64), (False, torch.int32)])
def test_step_decode_batch_slot_rules(cuda, B, tix, slot_dtype):
    """Decode batches (one new token per sequence), where the store computes
    its own slots beside the index build (one slot per lane group and token,
    at 200, 300 and 1,500 sequences): page ids outside the pool, a row
    outside the table, a sequence past its row's pages, a negative prior
    length and an int32 slot overflow must give the slots, pool and error
    bits the oracle gives."""
    rng = np.random.default_rng(7 + int(tix) + B)
    W, ps, E = 16, 16, 256
    R = B + 5 if tix else B
    pool_pages = max(6000, R * W + 16)
    P = (1 << 27) + 5 if slot_dtype == torch.int32 else pool_pages
    prior = rng.integers(0, W * ps - 1, B).astype(np.int32)
    new = np.ones(B, np.int32)
    # distinct page ids (two tokens on one slot in one call have no defined winner)
    table = rng.permutation(pool_pages)[:R * W].reshape(R, W).astype(np.int32)
    rows = rng.permutation(R)[:B].astype(np.int32) if tix else None
    r_of = (lambda i: rows[i]) if tix else (lambda i: i)
    prior[3] = W * ps + 20             # past its row's pages: no slot, no store
    prior[4] = -9                      # clamped to position 0
    table[r_of(5), prior[5] // ps] = P + 3       # page outside the pool
    table[r_of(6), prior[6] // ps] = -2          # negative page id
    if slot_dtype == torch.int32:
        table[r_of(7), prior[7] // ps] = (1 << 27)  # page * 16 + offset > INT_MAX: no int32 slot
    if tix:
        rows[8] = R + 100              # row outside the table
    S = pool_pages * ps + 16
    g = torch.Generator(device=cuda).manual_seed(1)
    k = torch.randn(2, B, E, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(2, B, E, generator=g, device=cuda).to(torch.bfloat16)
    kc = torch.randn(2, S, E, generator=g, device=cuda).to(torch.bfloat16)
    vc = torch.randn(2, S, E, generator=g, device=cuda).to(torch.bfloat16)
    want = orc.build_index(prior, new, table, ps, table_index=rows, num_pages=P,
                           slot_dtype=np.int64 if slot_dtype == torch.int64 else np.int32)
    want_k, want_v = host_bytes(kc).copy(), host_bytes(vc).copy()
    orc.store(host_bytes(k), host_bytes(v), want_k, want_v, want["slot_mapping"], num_slots=S)
    i32 = dict(dtype=torch.int32, device=cuda)
    out = yl.BatchIndex(torch.empty(B + 1, **i32), torch.empty(int(want["kv_indices"].size), **i32),
                        torch.empty(B, **i32), torch.empty(B + 1, **i32), torch.empty(B, dtype=slot_dtype, device=cuda))
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    yl.kv_step(_dev(prior, cuda), _dev(new, cuda), _dev(table, cuda), ps, k, v, kc, vc, out,
               table_index=None if rows is None else _dev(rows, cuda), num_pages=P, error_word=err)
    torch.cuda.synchronize()
    assert want["err"] & orc.PAGE_RANGE and int(err.item()) == want["err"]
    got = index_outputs(out)
    assert_index_equal(got, want)
    assert torch.equal(kc.view(torch.uint8).view(-1), torch.from_numpy(want_k.reshape(-1)).to(cuda))
    assert torch.equal(vc.view(torch.uint8).view(-1), torch.from_numpy(want_v.reshape(-1)).to(cuda))
