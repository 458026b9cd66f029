"""The CPU oracle that the GPU kernel tests compare against, checked against plain
dense PyTorch statements (hypothesis): paged attention over randomly permuted block
tables equals softmax attention over the gathered keys with GQA; the RMSNorm, RoPE
(both modes) and SiLU-gate statements match their textbook forms."""
import math

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200.ops import reference as ref


@settings(max_examples=40, deadline=None)
@given(seed=st.integers(0, 10 ** 6), S=st.integers(1, 3), Hkv=st.sampled_from([1, 2]), G=st.sampled_from([1, 2, 4]),
       D=st.sampled_from([16, 64]))
def test_paged_attention_oracle(seed, S, Hkv, G, D):
    g = torch.Generator().manual_seed(seed)
    lens = [int(torch.randint(1, 70, (1,), generator=g)) for _ in range(S)]
    mb = max((n + 15) // 16 for n in lens)
    nb = S * mb + 3
    perm = torch.randperm(nb, generator=g)[: S * mb].view(S, mb).to(torch.int32)
    kc = torch.randn(nb, Hkv, 16, D, generator=g)
    vc = torch.randn(nb, Hkv, 16, D, generator=g)
    # one query row per (sequence, context length) pair: the last row of each sequence and a middle one
    rows = [(s, n) for s, L in enumerate(lens) for n in sorted({L, max(1, L // 2)})]
    Hq = Hkv * G
    q = torch.randn(len(rows), Hq, D, generator=g)
    rseq = torch.tensor([s for s, _ in rows], dtype=torch.int32)
    rctx = torch.tensor([n for _, n in rows], dtype=torch.int32)
    scale = 1 / math.sqrt(D)
    got = ref.paged_attention(q, kc, vc, perm, rseq, rctx, Hq, scale)
    for i, (s, n) in enumerate(rows):
        pos = torch.arange(n)
        blk = perm[s, pos // 16].long()
        k = kc[blk, :, pos % 16]                    # [n, Hkv, D]
        v = vc[blk, :, pos % 16]
        k, v = k.repeat_interleave(G, 1), v.repeat_interleave(G, 1)
        p = torch.softmax(torch.einsum("hd,nhd->hn", q[i], k) * scale, -1)
        want = torch.einsum("hn,nhd->hd", p, v)
        assert torch.allclose(got[i].float().view(Hq, D), want, atol=1e-5), (s, n)


@settings(max_examples=40, deadline=None)
@given(seed=st.integers(0, 10 ** 6), T=st.integers(1, 9), D=st.sampled_from([8, 64]))
def test_norm_rope_act_oracles(seed, T, D):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, D, generator=g)
    w = torch.randn(D, generator=g)
    got = ref.rmsnorm(x, w, 1e-6).float()
    assert torch.allclose(got, x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w, atol=1e-5)
    gu = torch.randn(T, 2 * D, generator=g)
    assert torch.allclose(ref.silu_mul(gu).float(), torch.nn.functional.silu(gu[:, :D]) * gu[:, D:], atol=1e-5)
    H = 2
    xr = torch.randn(T, H, D, generator=g)
    pos = torch.randint(0, 5000, (T,), generator=g)
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2).float() / D))
    ang = pos[:, None].double() * inv.double()[None]         # [T, D/2]; float64 angles at large positions
    c, s_ = ang.cos().float()[:, None], ang.sin().float()[:, None]
    inter = ref.rope(xr, pos, inv, 0).float()                # pairs (2i, 2i+1)
    a, b = xr[..., 0::2], xr[..., 1::2]
    want = torch.stack([a * c - b * s_, a * s_ + b * c], -1).flatten(-2)
    assert torch.allclose(inter, want, atol=1e-4)
    half = ref.rope(xr, pos, inv, 1).float()                 # pairs (i, i + D/2)
    a, b = xr[..., : D // 2], xr[..., D // 2:]
    assert torch.allclose(half, torch.cat([a * c - b * s_, a * s_ + b * c], -1), atol=1e-4)


@settings(max_examples=30, deadline=None)
@given(seed=st.integers(0, 10 ** 6), k=st.integers(1, 80))
def test_dsa_oracles(seed, k):
    """Top-k keeps the k largest visible scores; sparse attention over every visible key
    equals dense paged attention."""
    from openmini_v1_b200.models import dsa
    g = torch.Generator().manual_seed(seed)
    lens = [int(torch.randint(1, 70, (1,), generator=g)) for _ in range(2)]
    S, mb = 2, 5
    nb = S * mb
    bt = torch.randperm(nb, generator=g).view(S, mb).to(torch.int32)
    kc = torch.randn(nb, 2, 16, 64, generator=g)
    vc = torch.randn(nb, 2, 16, 64, generator=g)
    rseq = torch.arange(S, dtype=torch.int32)
    rctx = torch.tensor(lens, dtype=torch.int32)
    scores = torch.randn(S, 80, generator=g)
    sel, n = dsa.topk_ref(scores, rctx, k)
    for r in range(S):
        c = lens[r]
        assert int(n[r]) == min(k, c)
        chosen = set(sel[r, :int(n[r])].tolist())
        assert all(0 <= j < c for j in chosen) and len(chosen) == int(n[r])
        if int(n[r]) < c:
            worst = min(float(scores[r, j]) for j in chosen)
            rest = [float(scores[r, j]) for j in range(c) if j not in chosen]
            assert worst >= max(rest)
    q = torch.randn(S, 4 * 64, generator=g)
    allk = torch.stack([torch.cat([torch.arange(c), torch.full((80 - c,), -1)]) for c in lens]).to(torch.int32)
    sp = dsa.sparse_attention_ref(q, kc, vc, bt, rseq, allk, rctx, 4, 0.125)
    dense = ref.paged_attention(q.view(S, 4, 64), kc, vc, bt, rseq, rctx, 4, 0.125)
    assert torch.allclose(sp.float().view(S, 4, 64), dense.float(), atol=1e-5)


@settings(max_examples=40, deadline=None)
@given(seed=st.integers(0, 10 ** 6), N=st.integers(1, 6), KB=st.integers(1, 4), mag=st.floats(1e-3, 50.0))
def test_weight_quantiser_error_bounds(seed, N, KB, mag):
    """4-bit blocks of 32 (scale = block max / -8): every value within one scale step
    (half a step except the clamped +8 end), and within bf16 rounding of the output;
    INT8 per row (scale = row max / 127): within half a step."""
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, 32 * KB, generator=g) * mag).bfloat16()
    q, d = ref.quantize_q4(w)
    back = ref.dequant_q4(q, d).float()
    wf = w.float()
    step = d.float().abs().repeat_interleave(32, 1)
    assert bool((back - wf).abs().le(step * 1.001 + back.abs() * 2 ** -8 + 1e-30).all())
    half = (back - wf).abs() <= step * 0.501 + back.abs() * 2 ** -8 + 1e-30
    assert half.float().mean() > 0.95
    qi, s = ref.quantize_int8(w)
    bi = ref.dequant_int8(qi, s).float()
    assert bool((bi - wf).abs().le(s[:, None] * 0.501 + bi.abs() * 2 ** -8 + 1e-30).all())
