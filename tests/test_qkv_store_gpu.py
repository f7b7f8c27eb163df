"""Fused Q/K RMSNorm + rotary embedding + K/V store on the GPU.

Checked three ways on seeded inputs: against the CPU oracle's restatement
of the unfused sequence, against a plain fp32 torch computation (tolerance
2e-2 absolute + 2e-2 relative), and against the reference's own norm kernel
(flashinfer QKRMSNorm, which src/layers/rsm_norm.cu:49 calls) followed by
flashinfer's rotary embedding.  V rows and every pool row the call must not
touch are bit-exact.  Q and K: the implementations differ only in fp32
rounding (the device's rsqrtf against 1/sqrt), which can move the rounded
norm output by one unit in the last place (ulp) of the 16-bit type; the
rotation a*c - b*s mixes two such values, so the bound is 2 ulp of the head
row's largest magnitude per element, with at most 1 % of elements differing.
Without rotation a single rounding separates them: at most 1 ulp per element.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import yllang_b200 as yl
from oracle import kvpath as orc

pytestmark = pytest.mark.gpu

ATOL = RTOL = 2e-2
DT = {torch.bfloat16: "bf16", torch.float16: "fp16"}


MANTISSA = {torch.bfloat16: 7, torch.float16: 10}


def _ordered(bits: np.ndarray) -> np.ndarray:
    u = bits.astype(np.int32) & 0xFFFF
    return np.where(u & 0x8000, -(u & 0x7FFF), u)


def assert_ulp_close(got: torch.Tensor, want: torch.Tensor, head_dim: int = 0, max_frac=0.01):
    """head_dim == 0: every element within 1 ulp of the 16-bit type.
    Otherwise every element within 2 ulp of its head row's largest magnitude.
    Either way at most max_frac of the elements differ."""
    got, want = got.detach().cpu().contiguous(), want.detach().cpu().contiguous()
    if head_dim == 0:
        d = np.abs(_ordered(got.view(torch.int16).numpy()) - _ordered(want.view(torch.int16).numpy()))
        assert d.max(initial=0) <= 1, f"max ulp diff {d.max()}"
        frac = (d != 0).mean()
    else:
        g, w = got.float().view(-1, head_dim), want.float().view(-1, head_dim)
        rowmax = w.abs().amax(-1, keepdim=True).clamp_min(1e-30)
        ulp = torch.exp2(torch.floor(torch.log2(rowmax)) - MANTISSA[want.dtype])
        err = (g - w).abs()
        assert bool((err <= 2 * ulp).all()), f"max error {float((err / ulp).max()):.2f} ulp of the row maximum"
        frac = float((g != w).float().mean())
    assert frac <= max_frac, f"{frac:.4f} of elements differ"


def _case(cuda, N, Hq, Hk, D, dtype, S, seed, fused_qkv=False):
    g = torch.Generator(device=cuda).manual_seed(seed)
    if fused_qkv:  # views of one [N, (Hq + 2Hk) * D] projection output
        qkv = torch.randn(N, (Hq + 2 * Hk) * D, generator=g, device=cuda).to(dtype)
        q = qkv[:, :Hq * D].view(N, Hq, D)
        k = qkv[:, Hq * D:(Hq + Hk) * D].view(N, Hk, D)
        v = qkv[:, (Hq + Hk) * D:].view(N, Hk, D)
    else:
        q = torch.randn(N, Hq, D, generator=g, device=cuda).to(dtype)
        k = torch.randn(N, Hk, D, generator=g, device=cuda).to(dtype)
        v = torch.randn(N, Hk, D, generator=g, device=cuda).to(dtype)
    qw = (1 + 0.2 * torch.randn(D, generator=g, device=cuda)).to(dtype)
    kw = (1 + 0.2 * torch.randn(D, generator=g, device=cuda)).to(dtype)
    k_cache = torch.randn(S, Hk * D, generator=g, device=cuda).to(dtype)
    v_cache = torch.randn(S, Hk * D, generator=g, device=cuda).to(dtype)
    slots = torch.randperm(S, generator=torch.Generator().manual_seed(seed))[:N].to(cuda)
    positions = torch.randint(0, 4096, (N,), generator=torch.Generator().manual_seed(seed + 1)).to(cuda)
    return q, k, v, qw, kw, k_cache, v_cache, slots, positions


def _oracle(q, k, v, k_cache, v_cache, slots, qw, kw, eps, cs, positions, interleaved, dtype):
    f = lambda t: None if t is None else t.float().cpu().numpy()
    Hk, D = k.shape[1], k.shape[2]
    kc = f(k_cache).reshape(-1, Hk, D).copy()
    vc = f(v_cache).reshape(-1, Hk, D).copy()
    q_out, err = orc.qkv_norm_rope_store(f(q), f(k), f(v), kc, vc, slots.cpu().numpy(), f(qw), f(kw), eps,
                                         None if cs is None else cs.cpu().numpy(),
                                         None if positions is None else positions.cpu().numpy(), interleaved,
                                         DT[dtype])
    t = lambda a: torch.from_numpy(a).to(dtype)
    return t(q_out), t(kc.reshape(k_cache.shape)), t(vc.reshape(v_cache.shape)), err


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("interleaved", [False, True])
def test_fused_matches_oracle(cuda, D, dtype, interleaved):
    N, Hq, Hk, S = 300, 8, 2, 1024
    q, k, v, qw, kw, k_cache, v_cache, slots, positions = _case(cuda, N, Hq, Hk, D, dtype, S, seed=D)
    cs = yl.rope_cos_sin_cache(4096, D, theta=1e6, device=cuda)
    want_q, want_k, want_v, bits = _oracle(q, k, v, k_cache, v_cache, slots, qw, kw, 1e-6, cs, positions,
                                           interleaved, dtype)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    q_out = yl.qkv_norm_rope_store(q, k, v, k_cache, v_cache, slots, q_weight=qw, k_weight=kw, eps=1e-6,
                                   cos_sin_cache=cs, positions=positions, interleaved=interleaved, error_word=err)
    torch.cuda.synchronize()
    assert bits == 0 and int(err.item()) == 0
    assert_ulp_close(q_out, want_q, D)
    assert_ulp_close(k_cache, want_k, D)  # written rows within the bound, the others untouched
    assert torch.equal(v_cache.cpu(), want_v)
    untouched = torch.ones(S, dtype=torch.bool)
    untouched[slots.cpu()] = False
    assert torch.equal(k_cache.cpu()[untouched], want_k[untouched])


@pytest.mark.parametrize("Hq,Hk,D", [(32, 8, 128), (12, 3, 128), (16, 4, 256), (8, 1, 64)])
def test_fused_large_batch_matches_oracle(cuda, Hq, Hk, D):
    """8192 tokens: enough chunks for the 8-head (4 at head_dim 256) chunk
    kernel, including partial chunks (12 Q heads, 3 KV heads)."""
    N, S = 8192, 16384
    q, k, v, qw, kw, k_cache, v_cache, slots, positions = _case(cuda, N, Hq, Hk, D, torch.bfloat16, S, seed=Hq + D)
    cs = yl.rope_cos_sin_cache(4096, D, theta=1e6, device=cuda)
    want_q, want_k, want_v, _ = _oracle(q, k, v, k_cache, v_cache, slots, qw, kw, 1e-6, cs, positions, False,
                                        torch.bfloat16)
    q_out = yl.qkv_norm_rope_store(q, k, v, k_cache, v_cache, slots, q_weight=qw, k_weight=kw, eps=1e-6,
                                   cos_sin_cache=cs, positions=positions)
    torch.cuda.synchronize()
    assert_ulp_close(q_out, want_q, D)
    assert_ulp_close(k_cache, want_k, D)
    assert torch.equal(v_cache.cpu(), want_v)


@pytest.mark.parametrize("norm,rope", [(False, False), (True, False), (False, True)])
def test_fused_stages_optional(cuda, norm, rope):
    N, Hq, Hk, D, S = 64, 4, 2, 128, 256
    q, k, v, qw, kw, k_cache, v_cache, slots, positions = _case(cuda, N, Hq, Hk, D, torch.bfloat16, S, seed=3)
    cs = yl.rope_cos_sin_cache(4096, D, device=cuda) if rope else None
    pos = positions if rope else None
    want_q, want_k, want_v, _ = _oracle(q, k, v, k_cache, v_cache, slots, qw if norm else None,
                                        kw if norm else None, 1e-6, cs, pos, False, torch.bfloat16)
    q_out = yl.qkv_norm_rope_store(q, k, v, k_cache, v_cache, slots, q_weight=qw if norm else None,
                                   k_weight=kw if norm else None, cos_sin_cache=cs, positions=pos)
    torch.cuda.synchronize()
    if not norm and not rope:  # a plain copy of Q and store of K/V: bit-exact
        assert torch.equal(q_out, q) and torch.equal(k_cache.cpu(), want_k)
    assert_ulp_close(q_out, want_q, D if rope else 0)
    assert_ulp_close(k_cache, want_k, D if rope else 0)
    assert torch.equal(v_cache.cpu(), want_v)


def test_fused_against_fp32_torch(cuda):
    """Qwen3-8B layer shape at decode (Hq 32, Hk 8, D 128), from one fused QKV
    projection, in place on q, against fp32 torch with no intermediate rounding."""
    N, Hq, Hk, D, S = 256, 32, 8, 128, 4096
    q, k, v, qw, kw, k_cache, v_cache, slots, positions = _case(cuda, N, Hq, Hk, D, torch.bfloat16, S, seed=9,
                                                                 fused_qkv=True)
    q0, k0 = q.float().clone(), k.float().clone()
    cs = yl.rope_cos_sin_cache(4096, D, theta=1e6, device=cuda)
    out = yl.qkv_norm_rope_store(q, k, v, k_cache, v_cache, slots, q_weight=qw, k_weight=kw, eps=1e-6,
                                 cos_sin_cache=cs, positions=positions, q_out=q)
    torch.cuda.synchronize()
    assert out.data_ptr() == q.data_ptr()

    def ref(x, w):
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
        c, s = cs[positions.long(), None, :D // 2], cs[positions.long(), None, D // 2:]
        a, b = x[..., :D // 2], x[..., D // 2:]
        return torch.cat([a * c - b * s, b * c + a * s], -1)

    torch.testing.assert_close(q.float(), ref(q0, qw), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(k_cache[slots.long()].view(N, Hk, D).float(), ref(k0, kw), atol=ATOL, rtol=RTOL)
    assert torch.equal(v_cache[slots.long()].view(N, Hk, D), v)


def test_fused_against_flashinfer_norm_and_rope(cuda):
    """The reference's norm kernel (flashinfer QKRMSNorm, CUDA build) then
    flashinfer's rotary embedding, then the store: the fused kernel agrees
    within one ulp."""
    from yllang_b200.attention import _flashinfer

    fi = _flashinfer()
    N, Hq, Hk, D, S = 512, 16, 4, 128, 2048
    q, k, v, qw, kw, k_cache, v_cache, slots, positions = _case(cuda, N, Hq, Hk, D, torch.bfloat16, S, seed=21)
    cs = yl.rope_cos_sin_cache(8192, D, theta=1e6, device=cuda)
    qn = fi.norm.rmsnorm(q.contiguous(), qw, eps=1e-6)
    kn = fi.norm.rmsnorm(k.contiguous(), kw, eps=1e-6)
    qr, kr = fi.rope.apply_rope_with_cos_sin_cache(positions, qn.view(N, Hq * D), kn.view(N, Hk * D), D, cs,
                                                   is_neox=True)
    kc2, vc2 = k_cache.clone(), v_cache.clone()
    yl.store_kv_cache(kr.view(N, Hk * D), v.reshape(N, Hk * D), kc2, vc2, slots)
    out = yl.qkv_norm_rope_store(q, k, v, k_cache, v_cache, slots, q_weight=qw, k_weight=kw, eps=1e-6,
                                 cos_sin_cache=cs, positions=positions)
    torch.cuda.synchronize()
    assert_ulp_close(out, qr.view(N, Hq, D), D)
    assert_ulp_close(k_cache, kc2, D)
    assert torch.equal(v_cache, vc2)


def test_fused_slot_and_position_errors(cuda):
    N, Hq, Hk, D, S = 16, 2, 2, 64, 64
    q, k, v, qw, kw, k_cache, v_cache, slots, positions = _case(cuda, N, Hq, Hk, D, torch.bfloat16, S, seed=5)
    cs = yl.rope_cos_sin_cache(4096, D, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    slots = slots.clone()
    positions = positions.clone()
    slots[3] = -1  # padding: skipped silently
    for case in ("padding", "errors"):
        if case == "errors":
            slots[5] = S + 3
            positions[7] = 4096
        want_q, want_k, want_v, bits = _oracle(q, k, v, k_cache, v_cache, slots, None, None, 1e-6, cs, positions,
                                               False, torch.bfloat16)
        q_out = torch.zeros_like(q)
        err.zero_()
        yl.qkv_norm_rope_store(q, k, v, k_cache, v_cache, slots, cos_sin_cache=cs, positions=positions, q_out=q_out,
                               error_word=err)
        torch.cuda.synchronize()
        keep = torch.ones(N, dtype=torch.bool)
        if case == "padding":
            assert bits == 0 and int(err.item()) == 0
        else:
            assert bits == orc.SLOT_RANGE | orc.POSITION_RANGE
            assert int(err.item()) == yl.DEVERR_SLOT_RANGE | yl.DEVERR_POSITION_RANGE
            assert int(q_out[7].abs().sum()) == 0  # token 7: nothing written
            keep[7] = False
        assert_ulp_close(q_out.cpu()[keep], want_q[keep], D)
        assert_ulp_close(k_cache, want_k, D)
        assert torch.equal(v_cache.cpu(), want_v)


def test_fused_with_index_build_positions(cuda):
    """Slots and positions of a ragged prefill + decode batch from the index
    build (position of new token t of sequence i = prior_len_i + t)."""
    ps, P, D, Hq, Hk = 16, 512, 128, 8, 2
    prior = np.array([0, 17, 100, 0, 5], np.int32)
    fresh = np.array([40, 1, 1, 77, 3], np.int32)
    W = 16
    pages = torch.randperm(P, generator=torch.Generator().manual_seed(1))[:5 * W].to(torch.int32).view(5, W)
    idx = yl.build_index(torch.from_numpy(prior).to(cuda), torch.from_numpy(fresh).to(cuda), pages.to(cuda), ps,
                         num_pages=P)
    positions = torch.from_numpy(np.concatenate([np.arange(p, p + n) for p, n in zip(prior, fresh)])).to(cuda)
    N = int(fresh.sum())
    q, k, v, qw, kw, _, _, _, _ = _case(cuda, N, Hq, Hk, D, torch.bfloat16, 1, seed=8)
    k_cache = torch.zeros(P * ps, Hk * D, dtype=torch.bfloat16, device=cuda)
    v_cache = torch.zeros_like(k_cache)
    cs = yl.rope_cos_sin_cache(1024, D, device=cuda)
    want_q, want_k, want_v, _ = _oracle(q, k, v, k_cache, v_cache, idx.slot_mapping, qw, kw, 1e-6, cs, positions,
                                        False, torch.bfloat16)
    out = yl.qkv_norm_rope_store(q, k, v, k_cache, v_cache, idx.slot_mapping, q_weight=qw, k_weight=kw,
                                 cos_sin_cache=cs, positions=positions)
    torch.cuda.synchronize()
    assert_ulp_close(out, want_q, D)
    assert_ulp_close(k_cache, want_k, D)
    assert torch.equal(v_cache.cpu(), want_v)


def test_fused_empty_and_argument_errors(cuda):
    q = torch.zeros(0, 4, 128, dtype=torch.bfloat16, device=cuda)
    k = torch.zeros(0, 2, 128, dtype=torch.bfloat16, device=cuda)
    kc = torch.zeros(8, 256, dtype=torch.bfloat16, device=cuda)
    out = yl.qkv_norm_rope_store(q, k, k, kc, kc.clone(), torch.zeros(0, dtype=torch.int64, device=cuda))
    assert out.shape == (0, 4, 128)
    q = torch.zeros(2, 4, 96, dtype=torch.bfloat16, device=cuda)
    k = torch.zeros(2, 2, 96, dtype=torch.bfloat16, device=cuda)
    kc = torch.zeros(8, 192, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(yl.KVPathError, match="UNSUPPORTED"):
        yl.qkv_norm_rope_store(q, k, k, kc, kc.clone(), torch.zeros(2, dtype=torch.int64, device=cuda))


def test_cpp_front_end_store_kv_norm_rope(cuda):
    """MHAKVCache::StoreKVNormRope on layer 1 of a paged pool (page size 16)
    against the Python entry point on the same layer's pool rows."""
    C = yl.load_extension()
    L, P, ps, Hq, Hk, D = 2, 64, 16, 8, 2, 128
    cache = C.MHAKVCache(L, P, Hk, D, C.KVCacheLayout.kLayerFirst, "cuda", torch.bfloat16, ps)
    N = 50
    q, k, v, qw, kw, _, _, slots, positions = _case(cuda, N, Hq, Hk, D, torch.bfloat16, P * ps, seed=31)
    cs = yl.rope_cos_sin_cache(4096, D, device=cuda)
    opts = C.QKNormRope()
    opts.q_weight, opts.k_weight, opts.eps = qw, kw, 1e-6
    opts.cos_sin_cache, opts.positions = cs, positions
    k_rows = torch.zeros(P * ps, Hk * D, dtype=torch.bfloat16, device=cuda)
    v_rows = torch.zeros_like(k_rows)
    want = yl.qkv_norm_rope_store(q, k, v, k_rows, v_rows, slots, q_weight=qw, k_weight=kw, eps=1e-6,
                                  cos_sin_cache=cs, positions=positions)
    got = cache.StoreKVNormRope(q, k, v, slots, 1, opts)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(cache.KCache(1).reshape(P * ps, Hk * D), k_rows)
    assert torch.equal(cache.VCache(1).reshape(P * ps, Hk * D), v_rows)
    assert float(cache.KCache(0).abs().sum()) == 0.0
    with pytest.raises(C.PanicError):
        cache.StoreKVNormRope(q.float(), k, v, slots, 1, opts)


@pytest.mark.parametrize("engine", ["register", "tma"])
def test_fused_engines_match(cuda, engine):
    """Every case above through one engine only: the register kernels (2- or
    8-head chunks) or the TMA-staged kernel, which otherwise only large
    batches reach (the engine is read once per process: run in a child)."""
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.abspath(__file__), "-k", "not engines_match"],
                       env=dict(os.environ, YL_QKV_ENGINE=engine), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
