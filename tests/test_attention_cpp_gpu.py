"""The C++ Attention layer (yllang::Attention, the reference's Attention of
src/include/layers/attention.h:22-68 made real) through the extension:
history stored into an MHAKVCache, then one step's projected QKV rows go
through Attention::Forward, which stores the step's K/V rows and runs
flashinfer's paged decode (every sequence adds one token) or causal paged
prefill over the pool with the step's page arrays.  Checked against a plain
fp32 attention over each sequence's contiguous history (tolerance 2e-2
absolute + 2e-2 relative, bf16 inputs, as the Python glue's test)."""
import numpy as np
import pytest
import torch

import yllang_b200 as yl

pytestmark = pytest.mark.gpu
C = yl.load_extension()
ATOL = RTOL = 2e-2


def _rmsnorm(x, w, eps):
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def _attend(q, keys, values, n_new):
    """fp32 causal attention of q [n_new, Hq, D] (the last n_new positions)
    over keys / values [n_all, Hk, D]."""
    Hq, Hk, D = q.shape[1], keys.shape[1], q.shape[2]
    kk = keys.float().repeat_interleave(Hq // Hk, dim=1)
    vv = values.float().repeat_interleave(Hq // Hk, dim=1)
    s = torch.einsum("thd,nhd->htn", q.float(), kk) / D ** 0.5
    n_all = kk.shape[0]
    dev = q.device
    allowed = torch.arange(n_all, device=dev)[None, :] <= (n_all - n_new + torch.arange(n_new, device=dev))[:, None]
    s = s.masked_fill(~allowed[None], float("-inf"))
    return torch.einsum("htn,nhd->thd", torch.softmax(s, dim=-1), vv)


def _setup(cuda, prior, fresh, Hq, Hk, D, ps, P, layers, layer, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    B = len(prior)
    W = int(max((int(p) + int(f) + ps - 1) // ps for p, f in zip(prior, fresh)))
    table = torch.randperm(P, generator=torch.Generator().manual_seed(seed + 1))[:B * W].to(torch.int32)
    table = table.view(B, W).to(cuda)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(cuda)
    cache = C.MHAKVCache(layers, P, Hk, D, C.KVCacheLayout.kLayerFirst, "cuda", torch.bfloat16, ps)
    hist_k = [torch.randn(int(n), Hk, D, generator=g, device=cuda).to(torch.bfloat16) for n in prior]
    hist_v = [torch.randn(int(n), Hk, D, generator=g, device=cuda).to(torch.bfloat16) for n in prior]
    pre = C.BuildBatchIndex(t(np.zeros(B)), t(prior), table, ps, num_pages=P)
    cache.StoreKV(torch.cat(hist_k), torch.cat(hist_v), pre.slot_mapping, layer)
    idx = C.BuildBatchIndex(t(prior), t(fresh), table, ps, num_pages=P)
    N = int(np.sum(fresh))
    qkv = torch.randn(N, (Hq + 2 * Hk) * D, generator=g, device=cuda).to(torch.bfloat16)
    return cache, hist_k, hist_v, idx, qkv


def _split(qkv, Hq, Hk, D):
    N = qkv.shape[0]
    q = qkv[:, :Hq * D].reshape(N, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hk) * D].reshape(N, Hk, D)
    v = qkv[:, (Hq + Hk) * D:].reshape(N, Hk, D)
    return q, k, v


@pytest.mark.parametrize("strided", [False, True])
def test_cpp_attention_decode(cuda, strided):
    Hq, Hk, D, ps, P = 32, 8, 128, 16, 2048
    rng = np.random.default_rng(5)
    prior = rng.integers(20, 300, 16).astype(np.int32)
    fresh = np.ones(16, np.int32)
    cache, hist_k, hist_v, idx, qkv = _setup(cuda, prior, fresh, Hq, Hk, D, ps, P, layers=2, layer=1, seed=0)
    if strided:  # rows of a wider buffer (a fused projection's output with extra columns)
        wide = torch.zeros(qkv.shape[0], qkv.shape[1] + 64, dtype=qkv.dtype, device=cuda)
        wide[:, :qkv.shape[1]] = qkv
        qkv = wide[:, :qkv.shape[1]]
    ctx = C.AttentionContext("cuda")
    ctx.Plan(idx, Hq, Hk, D, ps, torch.bfloat16)
    assert ctx.IsDecode()
    layer = C.Attention(1, Hq, Hk, D, cache)
    out = layer.Forward(qkv, ctx)
    torch.cuda.synchronize()
    assert out.shape == (16, Hq * D)
    q, k, v = _split(qkv, Hq, Hk, D)
    qo = idx.qo_indptr.tolist()
    for i in range(16):
        want = _attend(q[qo[i]:qo[i + 1]], torch.cat([hist_k[i], k[qo[i]:qo[i + 1]]]),
                       torch.cat([hist_v[i], v[qo[i]:qo[i + 1]]]), 1)
        torch.testing.assert_close(out[i].view(Hq, D).float(), want[0], atol=ATOL, rtol=RTOL)
    # the step's K/V rows are in the layer's pool at the step's slots, layer 0 untouched
    rows_k = cache.KCache(1).reshape(P * ps, Hk, D)
    assert torch.equal(rows_k[idx.slot_mapping.long()], k)
    assert float(cache.KCache(0).float().abs().sum()) == 0.0


def test_cpp_attention_prefill_through_the_step_context(cuda):
    """Chunked prefill mixed with decode tokens, through Forward(qkv) with the
    context set by SetAttentionContext."""
    Hq, Hk, D, ps, P = 16, 4, 128, 16, 1024
    prior = np.array([0, 37, 150, 1, 64, 300], np.int32)
    fresh = np.array([120, 1, 16, 200, 33, 5], np.int32)
    cache, hist_k, hist_v, idx, qkv = _setup(cuda, prior, fresh, Hq, Hk, D, ps, P, layers=1, layer=0, seed=1)
    ctx = C.AttentionContext("cuda")
    ctx.Plan(idx, Hq, Hk, D, ps, torch.bfloat16)
    assert not ctx.IsDecode()
    C.SetAttentionContext(ctx)
    try:
        out = C.Attention(0, Hq, Hk, D, cache).Forward(qkv)
    finally:
        C.SetAttentionContext(None)
    torch.cuda.synchronize()
    q, k, v = _split(qkv, Hq, Hk, D)
    qo = idx.qo_indptr.tolist()
    for i in range(len(prior)):
        want = _attend(q[qo[i]:qo[i + 1]], torch.cat([hist_k[i], k[qo[i]:qo[i + 1]]]),
                       torch.cat([hist_v[i], v[qo[i]:qo[i + 1]]]), int(fresh[i]))
        torch.testing.assert_close(out[qo[i]:qo[i + 1]].view(-1, Hq, D).float(), want, atol=ATOL, rtol=RTOL)


def test_cpp_attention_with_qk_norm(cuda):
    """A layer with per-head Q and K RMSNorm weights stores the normed K rows
    and attends with the normed q (the reference layer's qo_norm / k_norm)."""
    Hq, Hk, D, ps, P, eps = 16, 8, 128, 16, 1024, 1e-6
    rng = np.random.default_rng(9)
    prior = rng.integers(10, 200, 8).astype(np.int32)
    fresh = np.ones(8, np.int32)
    cache, hist_k, hist_v, idx, qkv = _setup(cuda, prior, fresh, Hq, Hk, D, ps, P, layers=1, layer=0, seed=2)
    g = torch.Generator(device=cuda).manual_seed(3)
    opts = C.QKNormRope()
    opts.q_weight = (1 + 0.1 * torch.randn(D, generator=g, device=cuda)).to(torch.bfloat16)
    opts.k_weight = (1 + 0.1 * torch.randn(D, generator=g, device=cuda)).to(torch.bfloat16)
    opts.eps = eps
    ctx = C.AttentionContext("cuda")
    ctx.Plan(idx, Hq, Hk, D, ps, torch.bfloat16)
    out = C.Attention(0, Hq, Hk, D, cache, opts).Forward(qkv, ctx)
    torch.cuda.synchronize()
    q, k, v = _split(qkv, Hq, Hk, D)
    qn = _rmsnorm(q, opts.q_weight, eps).to(torch.bfloat16)
    kn = _rmsnorm(k, opts.k_weight, eps).to(torch.bfloat16)
    for i in range(8):
        want = _attend(qn[i:i + 1], torch.cat([hist_k[i], kn[i:i + 1]]), torch.cat([hist_v[i], v[i:i + 1]]), 1)
        torch.testing.assert_close(out[i].view(Hq, D).float(), want[0], atol=ATOL, rtol=RTOL)


def _rope_neox(x, cs, positions):
    """Rotate-half rotary embedding by the [max_position, D] cos / sin cache."""
    D = x.shape[-1]
    c = cs[positions.long(), :D // 2][:, None, :]
    s = cs[positions.long(), D // 2:][:, None, :]
    x1, x2 = x[..., :D // 2].float(), x[..., D // 2:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def test_cpp_attention_with_norm_and_rotary_from_the_context(cuda):
    """Q/K RMSNorm then the rotary embedding at the step's positions (handed
    to the context by the step's driver), stored and attended."""
    Hq, Hk, D, ps, P, eps = 16, 8, 128, 16, 1024, 1e-6
    rng = np.random.default_rng(13)
    prior = rng.integers(10, 200, 8).astype(np.int32)
    fresh = np.ones(8, np.int32)
    cache, hist_k, hist_v, idx, qkv = _setup(cuda, prior, fresh, Hq, Hk, D, ps, P, layers=1, layer=0, seed=4)
    g = torch.Generator(device=cuda).manual_seed(5)
    opts = C.QKNormRope()
    opts.q_weight = (1 + 0.1 * torch.randn(D, generator=g, device=cuda)).to(torch.bfloat16)
    opts.k_weight = (1 + 0.1 * torch.randn(D, generator=g, device=cuda)).to(torch.bfloat16)
    opts.eps = eps
    opts.cos_sin_cache = yl.rope_cos_sin_cache(4096, D, theta=1e6, device=cuda)
    positions = torch.from_numpy(prior.astype(np.int64)).to(cuda)  # the new token's position
    ctx = C.AttentionContext("cuda")
    ctx.Plan(idx, Hq, Hk, D, ps, torch.bfloat16, positions)
    out = C.Attention(0, Hq, Hk, D, cache, opts).Forward(qkv, ctx)
    torch.cuda.synchronize()
    q, k, v = _split(qkv, Hq, Hk, D)
    qr = _rope_neox(_rmsnorm(q, opts.q_weight, eps), opts.cos_sin_cache, positions).to(torch.bfloat16)
    kr = _rope_neox(_rmsnorm(k, opts.k_weight, eps), opts.cos_sin_cache, positions).to(torch.bfloat16)
    for i in range(8):
        want = _attend(qr[i:i + 1], torch.cat([hist_k[i], kr[i:i + 1]]), torch.cat([hist_v[i], v[i:i + 1]]), 1)
        torch.testing.assert_close(out[i].view(Hq, D).float(), want[0], atol=ATOL, rtol=RTOL)
    ctx_no_pos = C.AttentionContext("cuda")
    ctx_no_pos.Plan(idx, Hq, Hk, D, ps, torch.bfloat16)
    with pytest.raises(RuntimeError, match="positions"):
        C.Attention(0, Hq, Hk, D, cache, opts).Forward(qkv, ctx_no_pos)


def test_cpp_attention_refusals(cuda):
    cache = C.MHAKVCache(1, 64, 8, 128, C.KVCacheLayout.kLayerFirst, "cuda", torch.bfloat16, 16)
    with pytest.raises(RuntimeError, match="layer_id"):
        C.Attention(3, 32, 8, 128, cache)
    with pytest.raises(RuntimeError, match="KV heads or head_dim"):
        C.Attention(0, 32, 4, 128, cache)
    layer = C.Attention(0, 32, 8, 128, cache)
    ctx = C.AttentionContext("cuda")
    with pytest.raises(RuntimeError, match="no plan"):
        layer.Forward(torch.zeros(1, 48 * 128, dtype=torch.bfloat16, device=cuda), ctx)
    C.SetAttentionContext(None)
    with pytest.raises(RuntimeError, match="no attention context"):
        layer.Forward(torch.zeros(1, 48 * 128, dtype=torch.bfloat16, device=cuda))
