"""Attention glue end to end: history stored through the step entry point,
one decode step stored and attended through flashinfer's paged decode over
the pool, checked against a plain fp32 attention over the contiguous
history (tolerance 2e-2 absolute + 2e-2 relative, bf16 inputs), and a
plain-torch consumer of the page arrays."""
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
