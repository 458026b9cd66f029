"""Experimental attention variants against full attention on the configurations
where they must agree, plus their own invariants."""
import torch

from openmini_v1_b200.models import attention_variants as av


def _qkv(T=70, H=4, Hkv=2, D=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(T, H, D, generator=g), torch.randn(T, Hkv, D, generator=g),
            torch.randn(T, Hkv, D, generator=g))


def test_nsa_branches():
    q, k, v = _qkv()
    full = av.full_attention(q, k, v)
    # every block selected and a window over the whole sequence: those branches are full attention
    o = av.nsa_attention(q, k, v, block=8, n_sel=100, window=1000)
    cmp_only = 3 * o - 2 * full  # = the compressed branch
    assert torch.isfinite(cmp_only).all()
    g = torch.zeros(4 * 3, 16)
    o2 = av.nsa_attention(q, k, v, block=8, n_sel=100, window=1000, gate_w=g)  # gates 0.5 each
    assert torch.allclose(o2, 0.5 * cmp_only + full, atol=1e-4)
    # a small selection budget differs from full attention but stays a convex combination
    o3 = av.nsa_attention(q, k, v, block=8, n_sel=2, window=8)
    assert not torch.allclose(o3, full, atol=1e-3)
    assert o3.abs().max() <= v.abs().max() + 1e-4


def test_kascade_reuse_and_sparse():
    q, k, v = _qkv(T=40)
    idx = av.kascade_indices(q, k, 1000)
    assert torch.allclose(av.sparse_attention(q, k, v, idx), av.full_attention(q, k, v), atol=1e-5)
    kc = av.KascadeCache(num_layers=8, anchor_interval=4, top_k=5)
    assert kc.anchors() == [0, 4]
    a0 = kc.indices(0, q, k)
    assert torch.equal(kc.indices(1, q * 3, k), a0) and kc.computed == 1
    assert (a0[10] >= 0).all() and (a0[10] <= 10).all() and (a0[2] >= 0).sum() == 3
    q2, k2, _ = _qkv(T=40, seed=1)
    kc.indices(4, q2, k2)
    u = av.KascadeCache(8, 4, 5, "union")
    u.indices(0, q, k)
    u.indices(4, q2, k2)
    m = u.indices(5, q2, k2)
    assert m.shape == (40, 5)


def test_tpa_factor_cache():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(12, 32, generator=g)
    H, D, R = 4, 8, 2
    wa, wb = torch.randn(R * H, 32, generator=g), torch.randn(R * D, 32, generator=g)
    K, kf = av.tpa_project(x, wa, wb, H, D, R)
    V, vf = av.tpa_project(x, wa * 0.5, wb, H, D, R)
    c = av.TPACache()
    c.append((kf[0][:5], kf[1][:5]), (vf[0][:5], vf[1][:5]))
    c.append((kf[0][5:], kf[1][5:]), (vf[0][5:], vf[1][5:]))
    k2, v2 = c.kv()
    assert torch.allclose(k2, K, atol=1e-5) and torch.allclose(v2, V, atol=1e-5)
    assert c.floats_per_token() == 2 * R * (H + D) < 2 * H * D + 1


def test_sinkhorn_doubly_stochastic():
    q, k, v = _qkv(T=16, H=2, Hkv=2)
    o, p = av.sinkhorn_attention(q, k, v, iters=50)
    assert torch.allclose(p.sum(-1), torch.ones(2, 16), atol=1e-5)
    assert torch.allclose(p.sum(-2), torch.ones(2, 16), atol=1e-3)
    assert o.shape == (16, 2, 16)


def test_attn_res_weights():
    g = torch.Generator().manual_seed(3)
    x0 = torch.randn(5, 8, generator=g)
    S = [torch.randn(5, 8, generator=g) for _ in range(3)]
    h, a = av.attn_res(x0, S, torch.zeros(8))
    assert torch.allclose(a, torch.full((3, 5), 1 / 3))
    assert torch.allclose(h, x0 + sum(S) / 3, atol=1e-6)
    _, a2 = av.attn_res(x0, S, torch.randn(8, generator=g) * 5)
    assert torch.allclose(a2.sum(0), torch.ones(5))


def test_linear_attention_chunked_equals_recurrent_and_ahn():
    q, k, v = _qkv(T=50)
    assert torch.allclose(av.linear_attention(q, k, v, chunk=16), av.linear_attention_recurrent(q, k, v), atol=1e-4)
    # window covering everything: AHN is exact local attention
    assert torch.allclose(av.ahn_attention(q, k, v, window=100), av.full_attention(q, k, v), atol=1e-5)
    o = av.ahn_attention(q, k, v, window=8, gate=torch.zeros(4))
    assert torch.isfinite(o).all() and not torch.allclose(o, av.full_attention(q, k, v), atol=1e-3)


def test_fp8_kv_roundtrip():
    g = torch.Generator().manual_seed(4)
    c = torch.randn(3, 2, 16, 64, generator=g).to(torch.bfloat16)
    codes, s = av.fp8_kv_quantize(c)
    assert codes.dtype == torch.float8_e4m3fn and s.shape == (3, 2)
    back = av.fp8_kv_dequantize(codes, s).float()
    rel = (back - c.float()).abs().max() / c.float().abs().max()
    assert rel < 0.07


def test_blockffn_sparse_equals_dense_statement():
    from openmini_v1_b200.models.moe_variants import BlockFFN
    f = BlockFFN(hidden=64, ffn=256, chunks=8, threshold=0.8, seed=1)
    x = torch.randn(30, 64, generator=torch.Generator().manual_seed(5))
    y = f(x)
    assert torch.allclose(y, f.dense_reference(x), atol=1e-5)
    assert 0.0 < f.last_density < 1.0  # some chunks skipped, some run
    f.thr = -1.0
    assert f(x).shape == (30, 64) and f.last_density == 1.0


def test_longcat_dual_branch():
    from openmini_v1_b200.models.moe_variants import LongCatDualBranch
    m = LongCatDualBranch(64, 128, 64, pivot=1000, width=100, skip_below=500, seed=2)
    x = torch.randn(10, 64, generator=torch.Generator().manual_seed(6))
    a, b = m.weights(100)
    assert b < 1e-3 and abs(a + b - 1) < 1e-9
    y_short = m(x, 100)
    assert m.aux_evaluated == 0
    y_long = m(x, 3000)
    assert m.aux_evaluated == 1 and not torch.allclose(y_short, y_long)
    a2, b2 = m.weights(3000)
    from openmini_v1_b200.models.moe_variants import _swiglu
    want = _swiglu(x, *m.main) * a2 + _swiglu(x, *m.aux) * b2
    assert torch.allclose(y_long, want, atol=1e-6)


def test_hp_pipeline_strategies():
    from openmini_v1_b200.models.hp_pipeline import HighPerfPipelineConfig, HighPerformancePipeline
    p = HighPerformancePipeline(HighPerfPipelineConfig(streaming_threshold=64, window=16, sinks=2))
    q, k, v = _qkv(T=40)
    o, s = p.forward(q, k, v)
    assert s == "flash" and torch.allclose(o, av.full_attention(q, k, v), atol=1e-5)
    q, k, v = _qkv(T=100)
    o, s = p.forward(q, k, v)
    assert s == "streaming"
    t = 80  # row 80 sees keys 0, 1 and 65..80
    keep = [0, 1] + list(range(65, 81))
    want = av.full_attention(q[t:t + 1], k[keep], v[keep], causal=False)
    assert torch.allclose(o[t], want[0], atol=1e-5)
    assert p.stats.by_strategy == {"flash": 1, "streaming": 1} and p.stats.calls == 2
