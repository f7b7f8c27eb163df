"""KV-head sharding across GPUs (tensor-parallel ranks).

The store and index build shard naturally by KV head with no exchange step:
rank g of G owns heads [g * H / G, (g + 1) * H / G) of every layer's pool (the
reference computes H_local = H / tp size, src/include/kvcache/mha_kvcache.h:45-46)
and stores its head slice of every new token under the same slot mapping.
The index build depends only on lengths and page ids, so every rank runs it
for the whole batch (replicated, a few microseconds) instead of sending it.
"""
from __future__ import annotations

import torch


def head_range(rank: int, world: int, num_kv_heads: int) -> tuple[int, int]:
    """[first, last) KV heads owned by `rank`; heads must divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def head_slice(kv: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """The rank's heads of K or V rows shaped [..., H, D], as [..., H_local * D]
    rows (a strided view when world > 1; the store takes row strides)."""
    h0, h1 = head_range(rank, world, kv.shape[-2])
    part = kv[..., h0:h1, :]
    return part.reshape(*part.shape[:-2], -1) if world == 1 else part.flatten(-2)


def max_over_ranks(value: float, group=None) -> float:
    """Largest `value` over the process group (timings are reported as the
    slowest rank's); the identity without an initialised group."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return value
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def sum_over_ranks(value: float, group=None) -> float:
    """Sum of `value` over the process group (bytes and tokens of all ranks)."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return value
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return float(t.item())


def gather_over_ranks(value: float, group=None) -> list[float]:
    """`value` of every rank of the process group, in rank order ([value]
    without an initialised group)."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return [value]
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    world = dist.get_world_size(group)
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t, group=group)
    return [float(x.item()) for x in out]
