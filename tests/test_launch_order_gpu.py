"""Stream order under programmatic launch.  The index build (and the step's
index build and store, and the allocator) are launched as programmatic
dependents of the kernel before them, and must still see every write that
kernel made: a torch kernel on the same stream rewrites the lengths, the
page table and the K/V rows immediately before each call, and the outputs
must be the oracle's for the rewritten inputs, call after call, with no
synchronisation in between."""
import numpy as np
import pytest
import torch

import yllang_b200 as yl
from _kvutil import assert_index_equal, index_outputs
from oracle import kvpath as orc
from yllang_b200 import workloads

pytestmark = pytest.mark.gpu


def test_index_build_sees_the_previous_kernels_writes(cuda):
    rng = np.random.default_rng(21)
    B, W, ps, P = 300, 24, 16, 8192
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    prior_d = torch.zeros(B, dtype=torch.int32, device=cuda)
    new_d = torch.zeros(B, dtype=torch.int32, device=cuda)
    table_d = torch.full((B, W), -1, dtype=torch.int32, device=cuda)
    for it in range(6):
        prior = rng.integers(0, (W - 2) * ps, B).astype(np.int32)
        new = (np.ones(B) if it % 2 == 0 else rng.integers(0, 2 * ps, B)).astype(np.int32)
        table = rng.permutation(P)[:B * W].astype(np.int32).reshape(B, W)
        src = [t(prior), t(new), t(table)]
        torch.cuda.synchronize()
        # the writes: elementwise kernels on the current stream, right before the call
        torch.add(src[0], 0, out=prior_d)
        torch.add(src[1], 0, out=new_d)
        torch.add(src[2], 0, out=table_d)
        want = orc.build_index(prior, new, table, ps, num_pages=P)
        idx = yl.build_index(prior_d, new_d, table_d, ps, num_pages=P, kv_indices_capacity=want["kv_indices"].size,
                             slot_capacity=want["slot_mapping"].size)
        got = index_outputs(idx)  # read back after this call, before the next rewrite
        torch.cuda.synchronize()
        assert_index_equal(got, want)


def test_step_sees_the_previous_kernels_writes(cuda):
    """A decode step whose K/V rows and page table a kernel rewrites just
    before it: the pool rows hold the new K/V at the slots of the new table."""
    b = workloads.llama3_decode(num_pages=4096, batch=200, layers=3)
    E = b.kv_heads * b.head_dim
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    g = torch.Generator(device=cuda).manual_seed(3)
    prior_d, new_d, table_d = t(b.prior_len), t(b.new_len), t(b.page_table)
    k = torch.zeros(b.layers, b.tokens, E, dtype=torch.bfloat16, device=cuda)
    v = torch.zeros_like(k)
    S = b.num_pages * b.page_size
    kc = torch.zeros(b.layers, S, E, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    out = yl.BatchIndex(torch.empty(b.batch + 1, dtype=torch.int32, device=cuda),
                        torch.empty(b.total_pages, dtype=torch.int32, device=cuda),
                        torch.empty(b.batch, dtype=torch.int32, device=cuda),
                        torch.empty(b.batch + 1, dtype=torch.int32, device=cuda),
                        torch.empty(b.tokens, dtype=torch.int64, device=cuda))
    rng = np.random.default_rng(5)
    for it in range(4):
        mapping = rng.permutation(b.num_pages).astype(np.int32)  # a bijection keeps written pages unique
        table = np.where(b.page_table >= 0, mapping[np.maximum(b.page_table, 0)], -1).astype(np.int32)
        kn = torch.randn(b.layers, b.tokens, E, generator=g, device=cuda).to(torch.bfloat16)
        vn = torch.randn(b.layers, b.tokens, E, generator=g, device=cuda).to(torch.bfloat16)
        tn = t(table)
        torch.cuda.synchronize()
        torch.add(tn, 0, out=table_d)            # the writes, right before the step
        torch.mul(kn, 1, out=k)
        torch.mul(vn, 1, out=v)
        yl.kv_step(prior_d, new_d, table_d, b.page_size, k, v, kc, vc, out, num_pages=b.num_pages)
        want = orc.build_index(b.prior_len, b.new_len, table, b.page_size, num_pages=b.num_pages)
        slots = torch.from_numpy(want["slot_mapping"]).to(cuda)
        torch.cuda.synchronize()
        assert torch.equal(out.slot_mapping.cpu(), torch.from_numpy(want["slot_mapping"]))
        for layer in range(b.layers):
            assert torch.equal(kc[layer].index_select(0, slots), kn[layer])
            assert torch.equal(vc[layer].index_select(0, slots), vn[layer])
