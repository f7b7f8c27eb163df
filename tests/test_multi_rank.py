"""Two ranks over gloo on CPU: the KV-head shard of the store.

Each rank stores its head slice of the same tokens into its own head-slice
pool (the CPU oracle stands in for the kernel); the slices gathered from both
ranks must equal one full-head store, every rank must move the same bytes
(weak scaling, no exchange on the data path), and the reported time is the
slowest rank's.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from yllang_b200 import sharding, workloads


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import kvpath as orc

        H, D, L = 8, 16, 3
        b = workloads.llama3_decode(num_pages=400, batch=24, kv_heads=H, layers=L, ctx_lo=16, ctx_hi=160)
        idx = orc.build_index(b.prior_len, b.new_len, b.page_table, b.page_size, num_pages=b.num_pages)
        S = b.num_pages * b.page_size
        g = torch.Generator().manual_seed(0)  # every rank sees the same tokens
        k = torch.randint(-2**15, 2**15, (L, b.tokens, H, D), generator=g, dtype=torch.int16)
        v = torch.randint(-2**15, 2**15, (L, b.tokens, H, D), generator=g, dtype=torch.int16)
        h0, h1 = sharding.head_range(rank, world, H)
        ks = sharding.head_slice(k, rank, world).contiguous().numpy()
        vs = sharding.head_slice(v, rank, world).contiguous().numpy()
        pool_k = np.zeros((L, S, (h1 - h0) * D), np.int16)
        pool_v = np.zeros_like(pool_k)
        copied, err = orc.store(ks, vs, pool_k, pool_v, idx["slot_mapping"], num_slots=S)
        assert err == 0
        moved = sharding.sum_over_ranks(float(ks.nbytes + vs.nbytes))
        mine = float(ks.nbytes + vs.nbytes)
        slowest = sharding.max_over_ranks(float(rank + 1))
        per_rank = sharding.gather_over_ranks(float(10 + rank))
        mine32 = torch.from_numpy(pool_k).view(torch.int32)  # gloo gathers no int16
        parts = [torch.zeros_like(mine32) for _ in range(world)]
        dist.all_gather(parts, mine32)
        parts = [p.view(torch.int16) for p in parts]
        if rank == 0:
            full_k = np.zeros((L, S, H * D), np.int16)
            full_v = np.zeros_like(full_k)
            orc.store(k.reshape(L, b.tokens, H * D).numpy(), v.reshape(L, b.tokens, H * D).numpy(), full_k, full_v,
                      idx["slot_mapping"], num_slots=S)
            gathered = torch.cat([p.view(L, S, -1, D) for p in parts], dim=2).reshape(L, S, H * D).numpy()
            np.save(os.path.join(out_dir, "ok.npy"),
                    np.array([np.array_equal(gathered, full_k), moved == world * mine, slowest == world,
                              per_rank == [10.0 + r for r in range(world)]]))
    finally:
        dist.destroy_process_group()


def test_head_shard_two_ranks(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    ok = np.load(tmp_path / "ok.npy")
    assert ok.tolist() == [True, True, True, True]


def test_head_range_rules():
    assert sharding.head_range(0, 1, 8) == (0, 8)
    assert [sharding.head_range(r, 4, 8) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        sharding.head_range(0, 3, 8)
    with pytest.raises(ValueError):
        sharding.head_range(2, 2, 8)
    x = torch.arange(2 * 3 * 8 * 4).view(2, 3, 8, 4)
    assert torch.equal(sharding.head_slice(x, 1, 2), x[:, :, 4:8, :].reshape(2, 3, 16))
    assert sharding.max_over_ranks(3.5) == 3.5  # no process group: identity
    assert sharding.gather_over_ranks(2.5) == [2.5]
