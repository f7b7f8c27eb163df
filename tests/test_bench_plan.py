"""The bench's host-side planning at every rank count the scaling run uses
(no GPU): per-rank batches, head slices, pool sizing and input rotation for
each workload, and the weak-scaling invariant that every rank of a G-GPU run
moves the bytes one GPU moves."""
import argparse
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_llama3_decode_weak_scaling_shapes(world):
    batches, desc = bench.make_batches("llama3_decode", world, 150e9, 2)
    b = batches[0]
    assert desc["scaling"] == "weak" and desc["global_batch"] == 256 * world
    assert b.batch == 256 * world and b.kv_heads == 8 // world and b.tokens == 256 * world
    assert b.store_bytes() == bench.make_batches("llama3_decode", 1, 150e9, 1)[0][0].store_bytes() + 8 * 256 * (world - 1)
    assert desc["pool_gb_per_gpu"] <= 150.0 + 1e-6
    # distinct destination slots within a set, and the page table covers every sequence's pages
    assert b.page_table.shape[0] == b.batch and b.page_table.max() < b.num_pages


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("name", ["ragged_prefill", "qwen72b_decode", "mixed_ps16_hd128"])
def test_other_workloads_plan(world, name):
    batches, desc = bench.make_batches(name, world, 150e9, 1)
    b = batches[0]
    assert b.kv_heads == 8 // world and desc["kv_heads_per_gpu"] == 8 // world
    assert b.row_bytes == b.kv_heads * b.head_dim * 2


def test_plan_rotation_exceeds_l2():
    args = argparse.Namespace(workload="llama3_decode", rotate=0, pool_gb=150.0)
    R, pool_bytes, per_set = bench.plan(args, 1, 180e9)
    assert R * per_set > 2 * bench.L2_BYTES and 0 < pool_bytes <= 150e9


def test_head_split_must_be_even():
    with pytest.raises(Exception):
        bench.make_batches("llama3_decode", 3, 150e9, 1)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_reference_arm_times_the_whole_job(world):
    """At N ranks the reference arm (rank 0's host cores) runs the whole job
    of our arm: the global batch of all ranks with every KV head, i.e. N
    times one rank's store bytes for the weak-scaling decode, and the same
    batch with every head for the strong-scaling Qwen2-72B decode."""
    whole, desc = bench.make_batches("llama3_decode", world, 150e9, 1, whole_job=True)
    rank, _ = bench.make_batches("llama3_decode", world, 150e9, 1)
    assert whole[0].batch == 256 * world and whole[0].kv_heads == 8 and desc["global_batch"] == 256 * world
    assert whole[0].tokens * whole[0].row_bytes == world * rank[0].tokens * rank[0].row_bytes
    q, _ = bench.make_batches("qwen72b_decode", world, 150e9, 1, whole_job=True)
    assert q[0].batch == 512 and q[0].kv_heads == 8
