"""Attention glue end to end: history stored through the store entry point,
one decode step (and one chunked-prefill step) stored and attended through
flashinfer's paged decode (prefill) over the pool, checked against a plain
fp32 attention over the contiguous history (tolerance 2e-2 absolute + 2e-2
relative, bf16 inputs), and a plain-torch consumer of the page arrays."""
import numpy as np
import pytest
import torch

import yllang_b200 as yl
from yllang_b200 import workloads

pytestmark = pytest.mark.gpu

ATOL = RTOL = 2e-2


def _reference(q, hist_k, hist_v):
    """fp32 attention of each sequence's q over its contiguous K/V history."""
    out = []
    for i, (k, v) in enumerate(zip(hist_k, hist_v)):
        Hq, Hk = q.shape[1], k.shape[1]
        kk = k.float().repeat_interleave(Hq // Hk, dim=1)
        vv = v.float().repeat_interleave(Hq // Hk, dim=1)
        s = torch.einsum("hd,nhd->hn", q[i].float(), kk) / q.shape[-1] ** 0.5
        out.append(torch.einsum("hn,nhd->hd", torch.softmax(s, dim=-1), vv))
    return torch.stack(out)


@pytest.mark.parametrize("head_dim", [128])
def test_decode_attention_over_stored_pool(cuda, head_dim):
    from yllang_b200.attention import PagedDecodeAttention, paged_decode_reference

    g = torch.Generator(device=cuda).manual_seed(0)
    B, Hq, Hk, ps = 16, 32, 8, 16
    b = workloads.llama3_decode(num_pages=2048, batch=B, kv_heads=Hk, layers=1, ctx_lo=20, ctx_hi=300)
    b.head_dim = head_dim
    P = b.num_pages
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    table = t(b.page_table)
    k_pages = torch.zeros(P, ps, Hk, head_dim, dtype=torch.bfloat16, device=cuda)
    v_pages = torch.zeros_like(k_pages)
    # history: positions [0, prior) of every sequence, stored as one prefill step
    hist_k = [torch.randn(int(n), Hk, head_dim, generator=g, device=cuda).to(torch.bfloat16) for n in b.prior_len]
    hist_v = [torch.randn(int(n), Hk, head_dim, generator=g, device=cuda).to(torch.bfloat16) for n in b.prior_len]
    zero = torch.zeros(B, dtype=torch.int32, device=cuda)
    pre = yl.build_index(zero, t(b.prior_len), table, ps, num_pages=P)
    yl.store_kv_cache(torch.cat(hist_k).view(-1, Hk * head_dim), torch.cat(hist_v).view(-1, Hk * head_dim),
                      k_pages.view(P * ps, -1), v_pages.view(P * ps, -1), pre.slot_mapping)
    # decode step: one new token per sequence
    idx = yl.build_index(t(b.prior_len), t(b.new_len), table, ps, num_pages=P)
    attn = PagedDecodeAttention(Hq, Hk, head_dim, ps, device=cuda)
    attn.plan(idx)
    q = torch.randn(B, Hq, head_dim, generator=g, device=cuda).to(torch.bfloat16)
    k_new = torch.randn(B, Hk, head_dim, generator=g, device=cuda).to(torch.bfloat16)
    v_new = torch.randn(B, Hk, head_dim, generator=g, device=cuda).to(torch.bfloat16)
    out = attn.forward(q, k_new, v_new, k_pages, v_pages)
    torch.cuda.synchronize()
    want = _reference(q, [torch.cat([h, k_new[i:i + 1]]) for i, h in enumerate(hist_k)],
                      [torch.cat([h, v_new[i:i + 1]]) for i, h in enumerate(hist_v)])
    torch.testing.assert_close(out.float(), want, atol=ATOL, rtol=RTOL)
    # the page arrays alone reconstruct the same history from the pool
    torch.testing.assert_close(paged_decode_reference(q, k_pages, v_pages, idx, ps), want, atol=1e-4, rtol=1e-4)


def test_prefill_attention_over_stored_pool(cuda):
    """Chunked prefill + decode in one batch: sequences with cached history get
    1..200 new tokens, each new token attends causally to its history and to
    the new tokens up to itself."""
    from yllang_b200.attention import PagedPrefillAttention

    g = torch.Generator(device=cuda).manual_seed(1)
    Hq, Hk, D, ps, P = 16, 4, 128, 16, 1024
    prior = np.array([0, 37, 150, 1, 64, 300], np.int32)
    fresh = np.array([120, 1, 16, 200, 33, 5], np.int32)
    B, W = len(prior), 64
    pages = torch.randperm(P, generator=torch.Generator().manual_seed(3))[:B * W].to(torch.int32).view(B, W).to(cuda)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    k_pages = torch.zeros(P, ps, Hk, D, dtype=torch.bfloat16, device=cuda)
    v_pages = torch.zeros_like(k_pages)
    hist_k = [torch.randn(int(n), Hk, D, generator=g, device=cuda).to(torch.bfloat16) for n in prior]
    hist_v = [torch.randn(int(n), Hk, D, generator=g, device=cuda).to(torch.bfloat16) for n in prior]
    pre = yl.build_index(t(np.zeros(B)), t(prior), pages, ps, num_pages=P)
    yl.store_kv_cache(torch.cat(hist_k).view(-1, Hk * D), torch.cat(hist_v).view(-1, Hk * D),
                      k_pages.view(P * ps, -1), v_pages.view(P * ps, -1), pre.slot_mapping)
    idx = yl.build_index(t(prior), t(fresh), pages, ps, num_pages=P)
    N = int(fresh.sum())
    q = torch.randn(N, Hq, D, generator=g, device=cuda).to(torch.bfloat16)
    k_new = torch.randn(N, Hk, D, generator=g, device=cuda).to(torch.bfloat16)
    v_new = torch.randn(N, Hk, D, generator=g, device=cuda).to(torch.bfloat16)
    attn = PagedPrefillAttention(Hq, Hk, D, ps, device=cuda)
    attn.plan(idx)
    out = attn.forward(q, k_new, v_new, k_pages, v_pages)
    torch.cuda.synchronize()
    qo = idx.qo_indptr.tolist()
    for i in range(B):
        kk = torch.cat([hist_k[i], k_new[qo[i]:qo[i + 1]]]).float().repeat_interleave(Hq // Hk, dim=1)
        vv = torch.cat([hist_v[i], v_new[qo[i]:qo[i + 1]]]).float().repeat_interleave(Hq // Hk, dim=1)
        qi = q[qo[i]:qo[i + 1]].float()
        s = torch.einsum("thd,nhd->htn", qi, kk) / D ** 0.5
        n_new, n_all = qi.shape[0], kk.shape[0]
        allowed = torch.arange(n_all, device=cuda)[None, :] <= (n_all - n_new + torch.arange(n_new, device=cuda))[:, None]
        s = s.masked_fill(~allowed[None], float("-inf"))
        want = torch.einsum("htn,nhd->thd", torch.softmax(s, dim=-1), vv)
        torch.testing.assert_close(out[qo[i]:qo[i + 1]].float(), want, atol=ATOL, rtol=RTOL)
