"""Helpers shared by the GPU parity tests: byte views of tensors and the
oracle run of the same store/index call."""
from __future__ import annotations

import numpy as np
import torch

from oracle import kvpath as orc


def host_bytes(t: torch.Tensor) -> np.ndarray:
    """Raw bytes of a tensor as a uint8 numpy array of shape [..., row_bytes]."""
    t = t.detach().contiguous().cpu()
    return t.view(torch.uint8).numpy()


def random_bytes(shape, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, shape, dtype=torch.uint8, generator=g)


def oracle_store(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 slots: torch.Tensor, num_slots: int = 0):
    """Oracle result of storing (k, v) into copies of the given caches.

    Works on the byte images of the tensors, so any dtype and any row
    stride is fine; returns (k_cache_bytes, v_cache_bytes, err)."""
    kb, vb = host_bytes(k), host_bytes(v)
    kcb, vcb = host_bytes(k_cache).copy(), host_bytes(v_cache).copy()
    _, err = orc.store(kb, vb, kcb, vcb, slots.cpu().numpy(), num_slots=num_slots)
    return kcb, vcb, err


def index_outputs(idx) -> dict:
    return {name: getattr(idx, name).cpu().numpy() for name in idx._fields}


def assert_index_equal(got: dict, want: dict):
    """Equal outputs; the ragged outputs are compared on their defined
    prefixes (entries past kv_indptr[B] / qo_indptr[B] are never written)."""
    n_idx = min(int(want["kv_indptr"][-1]), want["kv_indices"].size)
    n_slot = min(int(want["qo_indptr"][-1]), want["slot_mapping"].size)
    for name in ("kv_indptr", "kv_indices", "kv_last_page_len", "qo_indptr", "slot_mapping"):
        g, w = got[name], want[name]
        assert g.shape == w.shape, (name, g.shape, w.shape)
        if name == "kv_indices":
            g, w = g[:n_idx], w[:n_idx]
        elif name == "slot_mapping":
            g, w = g[:n_slot], w[:n_slot]
        if not np.array_equal(g, w):
            bad = np.nonzero(g != w)[0]
            raise AssertionError(f"{name}: {bad.size} mismatches, first at {bad[:5]}: got {g[bad[:5]]} want {w[bad[:5]]}")
