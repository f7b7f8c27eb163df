"""Seeded synthetic batches for the store + index path.

Each generator returns a `Batch` of per-sequence lengths and page-table rows
with the shapes of one serving workload; callers draw the K/V rows (N(0, 1)
cast to the K/V dtype, from a seeded torch generator).  Seeds: lengths from
numpy default_rng(seed_len=1), page ids from default_rng(seed_pages=2).  Page
tables are randomly fragmented: consecutive pages of a sequence are
unrelated pool pages.

Workloads (num_pages is chosen by the caller to fit its memory):
  cpu_ref         1 layer, 8 KV heads x 128, page 16; priors 17/33/64/100 + 1
                  decode token each, plus one 48-token prefill
  llama3_decode   32 layers, 8 x 128, page 16; 256 sequences, context
                  U[128, 8192], 1 new token each
  ragged_prefill  32 layers, 8 x 128, page 16; 64 prompts U[128, 4096], prior 0
  qwen72b_decode  80 layers, 8 x 128 split over tp ranks, page 16; 512
                  sequences, context U[512, 32768], 1 new token each
  mixed           4 layers, 8 heads, page in {1, 16, 64}, head_dim in
                  {64, 128, 256}; 128 decode sequences (context U[128, 8192])
                  + 8 prefill chunks of 512 tokens (prior U[0, 4096])

When the contexts need more pages than the pool holds (qwen72b_decode at
full context), pages that are only read alias other pool pages; the pages
written this step (those holding a sequence's new tokens) stay unique.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class Batch:
    name: str
    layers: int
    kv_heads: int  # KV heads stored on this GPU
    head_dim: int
    page_size: int
    num_pages: int
    prior_len: np.ndarray  # int32 [B]
    new_len: np.ndarray  # int32 [B]
    page_table: np.ndarray  # int32 [B, W], row i belongs to sequence i, unused entries -1
    dtype_bytes: int = 2
    info: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return int(self.prior_len.shape[0])

    @property
    def tokens(self) -> int:
        return int(self.new_len.sum())

    @property
    def row_bytes(self) -> int:
        return self.kv_heads * self.head_dim * self.dtype_bytes

    @property
    def pages_per_seq(self) -> np.ndarray:
        tot = self.prior_len.astype(np.int64) + self.new_len
        return (tot + self.page_size - 1) // self.page_size

    @property
    def total_pages(self) -> int:
        return int(self.pages_per_seq.sum())

    def store_bytes(self) -> int:
        """Algorithmic bytes of one step's store: read + write of every K and V row, plus the slots."""
        return self.tokens * self.layers * 2 * 2 * self.row_bytes + self.tokens * 8

    def step_bytes(self, slot_bytes: int = 8) -> int:
        """Algorithmic bytes of one fused step: every K/V row read and written
        once, plus the index build's inputs and outputs (the slots are
        computed, not read back)."""
        return self.tokens * self.layers * 2 * 2 * self.row_bytes + self.index_bytes(slot_bytes)

    def index_bytes(self, slot_bytes: int = 8) -> int:
        """Algorithmic bytes of one index build (lengths, page-table reads, all five outputs)."""
        B, nnz, N = self.batch, self.total_pages, self.tokens
        return 8 * B + 4 * nnz + 2 * 4 * (B + 1) + 4 * nnz + 4 * B + slot_bytes * N


def _page_table(pages_per_seq: np.ndarray, new_len: np.ndarray, prior_len: np.ndarray, page_size: int,
                num_pages: int, rng: np.random.Generator) -> np.ndarray:
    B = pages_per_seq.shape[0]
    W = int(pages_per_seq.max()) if B else 1
    table = np.full((B, max(W, 1)), -1, np.int32)
    need = int(pages_per_seq.sum())
    if need <= num_pages:
        ids = rng.permutation(num_pages)[:need].astype(np.int32)
        off = 0
        for i, n in enumerate(pages_per_seq):
            table[i, :n] = ids[off:off + n]
            off += n
        return table
    # Pool too small for every context: pages written this step are unique,
    # read-only pages alias random pool pages.
    first_written = prior_len // page_size
    written = int((pages_per_seq - first_written).sum())
    assert written <= num_pages, "pool cannot hold the pages written in one step"
    uniq = rng.permutation(num_pages)[:written].astype(np.int32)
    off = 0
    for i, n in enumerate(pages_per_seq):
        w0 = int(first_written[i])
        table[i, :w0] = rng.integers(0, num_pages, w0, dtype=np.int32)
        table[i, w0:n] = uniq[off:off + n - w0]
        off += n - w0
    return table


def cpu_ref(num_pages: int = 1024, seed_pages: int = 2) -> Batch:
    prior = np.array([17, 33, 64, 100, 0], np.int32)
    new = np.array([1, 1, 1, 1, 48], np.int32)
    ps = 16
    pps = (prior.astype(np.int64) + new + ps - 1) // ps
    rng = np.random.default_rng(seed_pages)
    return Batch("cpu_ref", 1, 8, 128, ps, num_pages, prior, new, _page_table(pps, new, prior, ps, num_pages, rng))


def llama3_decode(num_pages: int, batch: int = 256, kv_heads: int = 8, layers: int = 32, seed_len: int = 1,
                  seed_pages: int = 2, ctx_lo: int = 128, ctx_hi: int = 8192) -> Batch:
    rng = np.random.default_rng(seed_len)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, batch).astype(np.int32)
    prior = ctx - 1
    new = np.ones(batch, np.int32)
    ps = 16
    pps = (ctx.astype(np.int64) + ps - 1) // ps
    table = _page_table(pps, new, prior, ps, num_pages, np.random.default_rng(seed_pages))
    return Batch("llama3_decode", layers, kv_heads, 128, ps, num_pages, prior, new, table)


def ragged_prefill(num_pages: int, requests: int = 64, kv_heads: int = 8, layers: int = 32, seed_len: int = 1,
                   seed_pages: int = 2, lo: int = 128, hi: int = 4096) -> Batch:
    rng = np.random.default_rng(seed_len)
    new = rng.integers(lo, hi + 1, requests).astype(np.int32)
    prior = np.zeros(requests, np.int32)
    ps = 16
    pps = (new.astype(np.int64) + ps - 1) // ps
    table = _page_table(pps, new, prior, ps, num_pages, np.random.default_rng(seed_pages))
    return Batch("ragged_prefill", layers, kv_heads, 128, ps, num_pages, prior, new, table)


def qwen72b_decode(num_pages: int, tp: int = 1, batch: int = 512, layers: int = 80, seed_len: int = 1,
                   seed_pages: int = 2, ctx_lo: int = 512, ctx_hi: int = 32768) -> Batch:
    rng = np.random.default_rng(seed_len)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, batch).astype(np.int32)
    prior = ctx - 1
    new = np.ones(batch, np.int32)
    ps = 16
    pps = (ctx.astype(np.int64) + ps - 1) // ps
    table = _page_table(pps, new, prior, ps, num_pages, np.random.default_rng(seed_pages))
    return Batch("qwen72b_decode", layers, 8 // tp, 128, ps, num_pages, prior, new, table, info={"tp": tp})


def mixed(num_pages: int, page_size: int = 16, head_dim: int = 128, decode: int = 128, chunks: int = 8,
          chunk_len: int = 512, layers: int = 4, seed_len: int = 1, seed_pages: int = 2) -> Batch:
    rng = np.random.default_rng(seed_len)
    dctx = rng.integers(128, 8192 + 1, decode).astype(np.int32)
    cprior = rng.integers(0, 4096 + 1, chunks).astype(np.int32)
    prior = np.concatenate([dctx - 1, cprior]).astype(np.int32)
    new = np.concatenate([np.ones(decode, np.int32), np.full(chunks, chunk_len, np.int32)])
    pps = (prior.astype(np.int64) + new + page_size - 1) // page_size
    table = _page_table(pps, new, prior, page_size, num_pages, np.random.default_rng(seed_pages))
    return Batch(f"mixed_ps{page_size}_hd{head_dim}", layers, 8, head_dim, page_size, num_pages, prior, new, table)


def pool_pages_for(bytes_budget: int, layers: int, row_bytes: int, page_size: int) -> int:
    """Pages of a [2, L, P, page_size, row] pool that fit in bytes_budget."""
    return int(bytes_budget // (2 * layers * page_size * row_bytes))
