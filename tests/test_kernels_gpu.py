"""Numerics of every sm_100a kernel against the plain PyTorch fp32 statement
of the same op (``openmini_v1_b200.ops.reference``), seeded random inputs."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from openmini_v1_b200 import _native, ops
from openmini_v1_b200.models.quantize import Int8Weight, Q4Weight
from openmini_v1_b200.ops import reference as ref

DEV = "cuda"


def _rand(*shape, dtype=torch.bfloat16, std=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * std).to(dtype)


def _close(a, b, rtol=2e-2, atol=2e-2):
    """At most 0.1% of elements outside atol + rtol |b| (bf16 rounding of long dot
    products), and none outside 8x that bound (a wrong tile cannot hide in the 0.1%)."""
    a, b = a.float(), b.float()
    err = (a - b).abs()
    tol = atol + rtol * b.abs()
    bad = (err > tol).float().mean().item()
    worst = (err / tol).max().item()
    assert bad < 1e-3 and worst <= 8.0, f"max err {err.max().item():.4g}, frac bad {bad:.4g}, worst/tol {worst:.3g}"


def test_native_loaded():
    assert _native.have_C()
    assert "openmini_v1_b200" in _native.C().__file__


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (7, 1280, 8192), (32, 10240, 8192), (64, 2000, 520),
                                   (128, 512, 256), (129, 384, 192), (300, 1000, 520), (1024, 2048, 4096),
                                   (2048, 4096, 1024)])
def test_gemm(M, N, K):
    x = _rand(M, K, seed=1)
    w = _rand(N, K, std=0.05, seed=2)
    y = ops.linear(x, w)
    torch.cuda.synchronize()
    ops.check_status()
    _close(y, ref.linear(x, w))


@pytest.mark.parametrize("M,N,K", [(16, 4096, 4096), (512, 1024, 2048)])
def test_gemm_residual_inplace(M, N, K):
    x = _rand(M, K, seed=3)
    w = _rand(N, K, std=0.05, seed=4)
    h = _rand(M, N, seed=5)
    expect = ref.linear(x, w, h)
    ops.linear(x, w, out=h, resid=h)
    torch.cuda.synchronize()
    _close(h, expect)


@pytest.mark.parametrize("swap,splits", [(0, 1), (1, 1), (1, 4), (0, 3)])
def test_gemm_forced_paths(swap, splits):
    M, N, K = 96, 768, 1024
    x = _rand(M, K, seed=6)
    w = _rand(N, K, std=0.05, seed=7)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    c = ops.ctx(DEV)
    _native.C().gemm(x, w, out, None, c.workspace("gemm", 1 << 24), c.status, swap, splits)
    torch.cuda.synchronize()
    _close(out, ref.linear(x, w))


def test_quantize_roundtrip_matches_reference():
    w = _rand(256, 512, std=0.02, seed=8)
    q = Q4Weight.from_dense(w)
    qr, sr = ref.quantize_q4(w.cpu())
    qg, sg = q.parts()
    assert torch.equal(qg.cpu(), qr)
    assert torch.equal(sg.cpu(), sr)
    assert torch.equal(q.dequantize().cpu(), ref.dequant_q4(qr, sr))
    i8 = Int8Weight.from_dense(w)
    q8, s8 = ref.quantize_int8(w.cpu())
    assert (i8.qweight.cpu().int() - q8.int()).abs().max() <= 1
    torch.testing.assert_close(i8.scale.cpu(), s8)


@pytest.mark.parametrize("kind", ["q4", "int8"])
@pytest.mark.parametrize("M,N,K", [(1, 1280, 8192), (32, 10240, 1024), (64, 1000, 4096), (100, 768, 512),
                                   (256, 2048, 1024), (300, 1024, 2048), (1024, 4096, 1024)])
def test_gemm_weight_only_quant(kind, M, N, K):
    w = _rand(N, K, std=0.02, seed=9)
    qw = Q4Weight.from_dense(w) if kind == "q4" else Int8Weight.from_dense(w)
    x = _rand(M, K, seed=10)
    y = qw.linear(x)
    torch.cuda.synchronize()
    ops.check_status()
    _close(y, ref.linear(x, qw.dequantize()))
    h = _rand(M, N, seed=11)
    expect = ref.linear(x, qw.dequantize(), h)
    qw.linear(x, out=h, resid=h)
    torch.cuda.synchronize()
    _close(h, expect)


@pytest.mark.parametrize("D", [256, 4096, 8192])
def test_rmsnorm(D):
    x = _rand(37, D, seed=8)
    w = _rand(D, seed=9) + 1
    _close(ops.rmsnorm(x, w, 1e-5), ref.rmsnorm(x, w, 1e-5))
    d = _rand(37, D, seed=10)
    x2, x3 = x.clone(), x.clone()
    y = ops.rmsnorm(x2, w, 1e-5, delta=d)
    yr = ref.rmsnorm(x3, w, 1e-5, delta=d)
    _close(x2, x3, 1e-2, 1e-2)
    _close(y, yr)


def test_act_norm_misc():
    gu = _rand(33, 2 * 688, seed=11)
    _close(ops.silu_mul(gu), ref.silu_mul(gu))
    x = _rand(17, 1024, seed=12)
    _close(ops.gelu(x), ref.gelu(x))
    w, b = _rand(1024, seed=13), _rand(1024, seed=14)
    _close(ops.layernorm(x, w, b, 1e-5), ref.layernorm(x, w, b, 1e-5))
    _close(ops.softmax(x, 0.5), ref.softmax(x, 0.5), 1e-3, 1e-5)
    table = _rand(1000, 256, seed=15)
    ids = torch.randint(0, 1000, (50,), device=DEV, dtype=torch.int32)
    assert torch.equal(ops.embedding(ids, table), ref.embedding(ids, table))


def _paged_setup(S, Hkv, D, lens, nb, seed=0):
    g = torch.Generator().manual_seed(seed)
    kc = _rand(nb, Hkv, 16, D, seed=seed + 1)
    vc = _rand(nb, Hkv, 16, D, seed=seed + 2)
    mb = max((l + 15) // 16 for l in lens)
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(S, mb, dtype=torch.int32)
    o = 0
    for s, l in enumerate(lens):
        n = (l + 15) // 16
        bt[s, :n] = perm[o:o + n].to(torch.int32)
        o += n
    return kc, vc, bt.to(DEV)


@pytest.mark.parametrize("impl", ["tc", "simt"])
@pytest.mark.parametrize("Hq,Hkv,D", [(8, 1, 128), (4, 2, 64), (32, 32, 128), (40, 8, 128), (64, 8, 128),
                                      (16, 1, 128)])
def test_paged_attention_decode(Hq, Hkv, D, impl):
    if impl == "tc" and D != 128:
        pytest.skip("tensor-core kernel needs head_dim 128")
    lens = [1, 17, 300, 513, 1500, 2049] if Hq <= 40 else [1, 17, 300, 2049]
    S = len(lens)
    kc, vc, bt = _paged_setup(S, Hkv, D, lens, 400, seed=20)
    q = _rand(S, Hq, D, seed=21)
    rseq = torch.arange(S, dtype=torch.int32, device=DEV)
    rctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(D)
    o = ops.paged_attention(q, kc, vc, bt, rseq, rctx, Hq, scale, max_ctx=4096, impl=impl)
    torch.cuda.synchronize()
    ops.check_status()
    _close(o.view(S, Hq, D), ref.paged_attention(q, kc, vc, bt, rseq, rctx, Hq, scale))


@pytest.mark.parametrize("impl", ["tc", "simt"])
def test_paged_attention_prefill_rows(impl):
    Hq, Hkv, D = 8, 2, 128
    L = 700
    kc, vc, bt = _paged_setup(1, Hkv, D, [L], 64, seed=30)
    q = _rand(L, Hq, D, seed=31)
    rseq = torch.zeros(L, dtype=torch.int32, device=DEV)
    rctx = torch.arange(1, L + 1, dtype=torch.int32, device=DEV)
    o = ops.paged_attention(q, kc, vc, bt, rseq, rctx, Hq, 0.088, max_ctx=L, impl=impl)
    torch.cuda.synchronize()
    _close(o.view(L, Hq, D), ref.paged_attention(q, kc, vc, bt, rseq, rctx, Hq, 0.088))


@pytest.mark.parametrize("mode", [0, 1])
def test_rope_kv(mode):
    T, Hq, Hkv, D = 40, 8, 2, 128
    qkv = _rand(T, (Hq + 2 * Hkv) * D, seed=40)
    pos = torch.randint(0, 100000, (T,), dtype=torch.int32, device=DEV)
    slots = torch.randperm(64 * 16, device=DEV)[:T].to(torch.int32)
    slots[3] = -1
    kc = torch.zeros(64, Hkv, 16, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.clone(), vc.clone()
    inv = ref.inv_freq(D, 500000.0).to(DEV)
    q1 = qkv.clone()
    ops.rope_kv(q1, pos, slots, kc, vc, inv, Hq, Hkv, D, mode)
    q2 = qkv.clone()
    ref.rope_kv(q2, pos, slots, kc2, vc2, inv, Hq, Hkv, D, mode)
    torch.cuda.synchronize()
    _close(q1, q2, 1e-2, 1e-2)
    _close(kc, kc2, 1e-2, 1e-2)
    assert torch.equal(vc, vc2)


def test_sampler_greedy_and_topk1():
    B, V = 8, 128256
    lg = _rand(B, V, seed=50) * 3
    z = torch.zeros(B, device=DEV)
    tok, lp, _ = ops.sample(lg, z, torch.ones(B, device=DEV), torch.zeros(B, dtype=torch.int32, device=DEV),
                            torch.zeros(B, 2, dtype=torch.int64, device=DEV))
    assert torch.equal(tok.long(), lg.float().argmax(-1))
    tok2, _, _ = ops.sample(lg, torch.full((B,), 0.7, device=DEV), torch.ones(B, device=DEV),
                            torch.ones(B, dtype=torch.int32, device=DEV),
                            torch.randint(0, 1 << 40, (B, 2), device=DEV))
    assert torch.equal(tok2.long(), lg.float().argmax(-1))


def test_sampler_matches_reference():
    B, V = 6, 32000
    lg = _rand(B, V, seed=51, dtype=torch.float32) * 2
    temp = torch.tensor([0.7, 1.0, 0.5, 1.3, 0.7, 0.9], device=DEV)
    top_p = torch.tensor([0.9, 0.5, 1.0, 0.95, 0.3, 0.8], device=DEV)
    top_k = torch.tensor([0, 50, 20, 0, 0, 1000], dtype=torch.int32, device=DEV)
    rng = torch.tensor([[11, 0], [12, 5], [13, 7], [14, 1], [15, 2], [16, 3]], dtype=torch.int64, device=DEV)
    tok, lp, mask = ops.sample(lg, temp, top_p, top_k, rng, want_mask=True)
    rt, rlp, rm = ref.sample(lg.cpu(), temp.cpu(), top_p.cpu(), top_k.cpu(), rng.cpu())
    gm = ref.unpack_mask(mask.cpu(), V)
    diff = (gm ^ rm).sum(-1)  # kept sets equal up to float-summation order at the cut-off
    assert int(diff.max()) <= 2, diff
    assert (tok.cpu() == rt).float().mean() >= 5 / 6
    torch.testing.assert_close(lp.cpu(), rlp, rtol=1e-3, atol=1e-3)
    for b in range(B):
        assert gm[b, int(tok[b])]


def test_sampler_distribution():
    V = 64
    lg = torch.full((1, V), -30.0, device=DEV)
    lg[0, :4] = torch.log(torch.tensor([0.1, 0.2, 0.3, 0.4], device=DEV))
    n = 4000
    lgb = lg.expand(n, V).contiguous()
    rng = torch.stack([torch.arange(n, device=DEV), torch.zeros(n, dtype=torch.int64, device=DEV)], 1).contiguous()
    tok, _, _ = ops.sample(lgb, torch.ones(n, device=DEV), torch.ones(n, device=DEV),
                           torch.zeros(n, dtype=torch.int32, device=DEV), rng)
    freq = torch.bincount(tok.long().cpu(), minlength=V)[:4].float() / n
    assert torch.allclose(freq, torch.tensor([0.1, 0.2, 0.3, 0.4]), atol=0.03), freq


def test_repetition_penalty():
    lg = _rand(2, 1000, seed=60, dtype=torch.float32)
    prev = torch.tensor([[1, 5, 5, -1], [7, 8, 9, 10]], dtype=torch.int32, device=DEV)
    pen = torch.tensor([1.3, 0.8], device=DEV)
    a = ops.repetition_penalty(lg.clone(), prev, pen)
    b = ref.repetition_penalty(lg.clone().cpu(), prev.cpu(), pen.cpu())
    torch.testing.assert_close(a.cpu(), b)


def test_dsa_kernels():
    from openmini_v1_b200.models import dsa
    rows, H, L = 5, 4, 1500
    lens = [1500, 1024, 700, 1, 1300]
    nb = 320
    icache = _rand(nb, 16, 64, seed=70)
    kc, vc, bt = _paged_setup(rows, 2, 128, lens, nb, seed=71)
    qi = _rand(rows, H * 64, seed=72)
    wi = torch.rand(rows, H, device=DEV)
    rseq = torch.arange(rows, dtype=torch.int32, device=DEV)
    rctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    c = ops.ctx(DEV)
    scores = torch.empty(rows, L, device=DEV)
    _native.C().dsa_scores(qi, wi, H, icache, bt, rseq, rctx, scores, c.status)
    sref = dsa.index_scores_ref(qi.cpu(), wi.cpu(), icache.cpu(), bt.cpu(), rseq.cpu(), rctx.cpu(), H, L)
    fin = torch.isfinite(sref)
    torch.testing.assert_close(scores.cpu()[fin], sref[fin], rtol=1e-3, atol=1e-3)
    k = 512
    sel = torch.empty(rows, k, dtype=torch.int32, device=DEV)
    n = torch.empty(rows, dtype=torch.int32, device=DEV)
    _native.C().dsa_topk(scores, rctx, k, sel, n)
    iref, nref = dsa.topk_ref(scores.cpu(), rctx.cpu(), k)
    assert torch.equal(n.cpu(), nref)
    for r in range(rows):
        assert set(sel[r, :n[r]].tolist()) == set(iref[r, :nref[r]].tolist())
    Hq = 8
    q = _rand(rows, Hq * 128, seed=73)
    out = torch.empty(rows, Hq * 128, dtype=torch.bfloat16, device=DEV)
    _native.C().dsa_attention(q, kc, vc, bt, rseq, sel, n, out, Hq, 0.088)
    oref = dsa.sparse_attention_ref(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), rseq.cpu(), sel.cpu(), n.cpu(), Hq, 0.088)
    _close(out.cpu(), oref)


@pytest.mark.parametrize("Hq,Hkv,qstd", [(8, 1, 1.0), (64, 8, 1.0), (4, 4, 6.0)])
def test_flash_prefill(Hq, Hkv, qstd):
    from openmini_v1_b200.engine.engine import LLMEngine
    chunks = [(0, 300), (200, 150), (0, 1), (1000, 129), (0, 1200)]  # (cached prefix, new rows)
    lens = [s + n for s, n in chunks]
    S = len(chunks)
    nb = sum((l + 15) // 16 for l in lens) + 8
    kc, vc, bt = _paged_setup(S, Hkv, 128, lens, nb, seed=80)
    T = sum(n for _, n in chunks)
    qkv = _rand(T, (Hq + 2 * Hkv) * 128, std=qstd, seed=81)
    rseq = torch.cat([torch.full((n,), i, dtype=torch.int32) for i, (_, n) in enumerate(chunks)]).to(DEV)
    rctx = torch.cat([torch.arange(s + 1, s + n + 1, dtype=torch.int32) for s, n in chunks]).to(DEV)

    class _C:
        def __init__(self, s, n):
            self.start, self.end = s, s + n

    class _SO:
        kind = "prefill"

    tiles = LLMEngine._prefill_tiles(_SO, [_C(s, n) for s, n in chunks], T)
    tiles = torch.tensor(tiles, dtype=torch.int32, device=DEV)
    out = ops.flash_prefill(qkv, kc, vc, bt, rseq, rctx, tiles, Hq, 1 / math.sqrt(128))
    ops.check_status()
    want = ref.paged_attention(qkv.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), rseq.cpu(), rctx.cpu(), Hq,
                               1 / math.sqrt(128))
    _close(out.cpu(), want.reshape(T, -1))


@pytest.mark.parametrize("T,E,k,forced", [(37, 8, 2, False), (300, 16, 2, False), (5, 4, 3, True)])
def test_moe_device_path(T, E, k, forced):
    from types import SimpleNamespace
    from openmini_v1_b200.models import moe
    D, F = 256, 128
    x = _rand(T, D, seed=90)
    L = {"router": _rand(E, D, std=0.2, seed=91),
         "experts_gate_up": [_rand(2 * F, D, std=0.06, seed=100 + e) for e in range(E)],
         "experts_down": [_rand(D, F, std=0.06, seed=200 + e) for e in range(E)]}
    model = SimpleNamespace(cfg=SimpleNamespace(moe=SimpleNamespace(top_k=k, num_experts=E, expert_ffn=F)))
    fr = {0: torch.randint(0, E, (T, k), device=DEV, dtype=torch.int32)} if forced else None
    fb = SimpleNamespace(forced_routing=fr, record_routing={})
    out = moe.moe_forward_device(model, 0, L, x, fb)
    ops.check_status()
    # fp32 statement of the same op
    lg = (x.float() @ L["router"].float().t()).bfloat16().float()
    if forced:
        ids = fr[0].long()
    else:
        # The router logits come from the tcgen05 GEMM rounded to bf16; another summation
        # order can move a near-tie by one bf16 ulp, so the kernel's choice is accepted when
        # its logits match the fp32 top-k values to within that rounding.
        ids = fb.record_routing[0].long()
        top, _ = torch.topk(lg, k, dim=-1)
        torch.testing.assert_close(lg.gather(1, ids), top, rtol=1.6e-2, atol=1e-2)
    sel = lg.gather(1, ids)
    w = torch.softmax(sel, -1)
    want = torch.zeros(T, D, device=DEV)
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            gu = x[t].float() @ L["experts_gate_up"][e].float().t()
            a = torch.nn.functional.silu(gu[:F]) * gu[F:]
            want[t] += w[t, j] * (a.bfloat16().float() @ L["experts_down"][e].float().t())
    _close(out, want)


@pytest.mark.parametrize("kind", ["bf16", "q4"])
@pytest.mark.parametrize("T,splits", [(6, 0), (6, 3), (256, 0)])
def test_gemm_peer_output(kind, T, splits):
    """Peer-output GEMM (the fused GEMM -> reduce-scatter store path) with two emulated
    ranks whose buffers both live on this GPU: rows [0, T/2) land in buffer 0 and rows
    [T/2, T) in buffer 1, each in slot `rank` of the partials region, and the last CTA
    bumps the epoch and writes ready[rank] in both buffers."""
    from openmini_v1_b200.models.quantize import Q4Weight
    D, K, W, rank = 512, 1024, 2, 1
    x = _rand(T, K, seed=300)
    w = _rand(D, K, std=0.05, seed=301)
    wt = Q4Weight.from_dense(w) if kind == "q4" else w
    rows_own = T // W
    off = 256
    bufs = [torch.zeros(off + T * D * 2 + 1024, dtype=torch.uint8, device=DEV) for _ in range(W)]
    peer = [off, rows_own, rank] + [b.data_ptr() for b in bufs]
    c = ops.ctx(DEV)
    ws = c.workspace("gemm", ops.GEMM_WS_FLOATS)
    dummy = torch.empty(T, D, dtype=torch.bfloat16, device=DEV)
    want = torch.empty(T, D, dtype=torch.bfloat16, device=DEV)
    kw = {"sem": c.semaphores()} if kind == "q4" and splits == 0 else {}  # stream-K decode kernel
    if kind == "q4":  # the same launch plan without peer output
        _native.C().gemm_wq(x, wt.tiles, None, 0, want, None, ws, c.status, force_splits=splits, **kw)
    else:
        _native.C().gemm(x, wt, want, None, ws, c.status, force_splits=splits)
    torch.testing.assert_close(want.float(), x.float() @ (wt.dequantize() if kind == "q4" else wt).float().t(),
                               rtol=2e-2, atol=2e-2)
    for rep in range(2):
        if kind == "q4":
            _native.C().gemm_wq(x, wt.tiles, None, 0, dummy, None, ws, c.status, force_splits=splits, peer=peer,
                                **kw)
        else:
            _native.C().gemm(x, wt, dummy, None, ws, c.status, force_splits=splits, peer=peer)
        torch.cuda.synchronize()
        ops.check_status()
        for o in range(W):
            slots = bufs[o][off:off + W * rows_own * D * 2].view(torch.bfloat16).view(W, rows_own, D)
            # (a SWAP-mode peer GEMM may take the split-K route: other summation order)
            torch.testing.assert_close(slots[rank].float(), want[o * rows_own:(o + 1) * rows_own].float(),
                                       rtol=1e-2, atol=1e-2)
        ctrl = bufs[rank][:256].view(torch.int32)
        assert int(ctrl[32]) == rep + 1  # epoch (byte 128) of the publishing rank
        for o in range(W):
            assert int(bufs[o][:256].view(torch.int32)[rank]) == rep + 1  # ready[rank] on every rank
        assert int(ctrl[34]) == 0  # GEMM CTA ticket (byte 136) reset


def test_flash_prefill_lse_and_ring_merge():
    """The prefill kernel's log-sum-exp output, and the ring-attention merge of per-chunk
    partials run through it (one GPU, chunks emulating 3 context-parallel ranks), against
    fp32 causal attention over the whole sequence."""
    from openmini_v1_b200.parallel.ring_attention import _attend_cpu, attend, merge
    T, H, Hkv, D = 3 * 160, 8, 2, 128
    q = _rand(T, H, D, seed=400)
    k = _rand(T, Hkv, D, seed=401)
    v = _rand(T, Hkv, D, seed=402)
    sc = 1 / math.sqrt(D)
    want, wlse = _attend_cpu(q.cpu(), k.cpu(), v.cpu(), sc, causal=True)
    o, l = attend(q, k, v, sc, causal=True)
    ops.check_status()
    _close(o.cpu(), want)
    torch.testing.assert_close(l.cpu(), wlse, rtol=1e-3, atol=2e-2)
    C = T // 3
    for r in range(3):
        sl = slice(r * C, (r + 1) * C)
        out, lse = attend(q[sl], k[sl], v[sl], sc, causal=True)
        for s in range(r):
            o_s, l_s = attend(q[sl], k[s * C:(s + 1) * C], v[s * C:(s + 1) * C], sc, causal=False)
            out, lse = merge(out, lse, o_s, l_s)
        _close(out.cpu(), want[sl])


def test_sliding_window_attention_gpu():
    """Window attention (device index lists + sparse-gather kernel) against the CPU path."""
    from types import SimpleNamespace
    from openmini_v1_b200.models.window import window_attention
    Hq, Hkv, D, W = 8, 2, 128, 64
    lens = [1, 40, 300, 700]
    S = len(lens)
    kc, vc, bt = _paged_setup(S, Hkv, D, lens, 80, seed=500)
    q = _rand(S, Hq * D, seed=501)
    fb = SimpleNamespace(max_ctx=max(lens), block_tables=bt, row_seq=torch.arange(S, dtype=torch.int32, device=DEV),
                         row_ctx=torch.tensor(lens, dtype=torch.int32, device=DEV), prefill_tiles=None)
    m = SimpleNamespace(hq=Hq, hd=D, scale=1 / math.sqrt(D))
    out = window_attention(m, q, kc, vc, fb, W)
    ops.check_status()
    fbc = SimpleNamespace(max_ctx=fb.max_ctx, block_tables=bt.cpu(), row_seq=fb.row_seq.cpu(), row_ctx=fb.row_ctx.cpu(),
                          prefill_tiles=None)
    _close(out.cpu(), window_attention(m, q.cpu(), kc.cpu(), vc.cpu(), fbc, W))


def test_vision_encoder_gpu():
    """ViT encoder on the GPU kernels (GEMM, LayerNorm, GELU, bidirectional FlashAttention)
    against the same encoder's fp32 CPU statement."""
    from openmini_v1_b200.models.vision import VisionConfig, VisionEncoder, preprocess
    cfg = VisionConfig(image_size=224, patch_size=16, hidden_size=1024, num_layers=2, num_heads=8, mlp_size=2048,
                       lm_hidden=512)
    enc = VisionEncoder(cfg, device=DEV, seed=2)
    cpu = VisionEncoder(cfg, device="cpu", seed=2)
    img = torch.rand(224, 224, 3, generator=torch.Generator().manual_seed(3))
    p = preprocess(img, cfg)[0]
    got = enc.encode(p)
    ops.check_status()
    _close(got.cpu(), cpu.encode(p), rtol=5e-2, atol=5e-2)


@pytest.mark.parametrize("kind", ["q4", "int8"])
@pytest.mark.parametrize("M,N,K", [(1, 1000, 2048), (7, 1536, 2048), (32, 10240, 1024), (33, 384, 8192),
                                   (64, 28672 // 8, 8192), (100, 1024, 4096), (128, 8192, 3584),
                                   (129, 1280, 8192), (200, 1000, 2048), (256, 7168, 8192)])
def test_gemm_wq_streamk_decode(kind, M, N, K):
    """Stream-K TMEM-operand decode kernel (M <= 256; two token halves above 128) against the fp32 statement and
    against the shared-memory-operand kernel (forced split-K route), with a residual,
    on repeated launches: the per-group counters must come back zeroed."""
    x = _rand(M, K, seed=600)
    w = _rand(N, K, std=0.05, seed=601)
    r = _rand(M, N, seed=602)
    wt = Q4Weight.from_dense(w) if kind == "q4" else Int8Weight.from_dense(w)
    sc = None if kind == "q4" else wt.scale
    c = ops.ctx(DEV)
    ws = c.workspace("gemm", ops.GEMM_WS_FLOATS)
    sem = c.semaphores()
    other = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    _native.C().gemm_wq(x, wt.tiles, sc, wt.qtype, other, r, ws, c.status, force_splits=2)
    expect = ref.linear(x, wt.dequantize(), r)
    first = None
    for _ in range(4):
        got = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
        _native.C().gemm_wq(x, wt.tiles, sc, wt.qtype, got, r, ws, c.status, sem=sem)
        torch.cuda.synchronize()
        ops.check_status()
        _close(got, expect)
        _close(got, other, rtol=1e-2, atol=1e-2)
        # the partial sums are added in CTA order: repeated launches agree bit for bit
        # (a shared-memory slot overwritten before it was read once broke this for INT8)
        if first is None:
            first = got
        else:
            assert torch.equal(got, first)
    assert int(sem.abs().sum()) == 0


@pytest.mark.parametrize("impl", ["simt", "tc"])
def test_paged_attention_context_bounds(impl):
    """A row whose context is longer than its block-table row (or than max_ctx) is
    reported through the status word (bounds error) instead of reading past the table
    or silently dropping keys."""
    Hq, Hkv, D = 16, 2, 128
    kc = _rand(64, Hkv, 16, D, seed=700)
    vc = _rand(64, Hkv, 16, D, seed=701)
    bt = torch.arange(8, dtype=torch.int32, device=DEV).view(2, 4)
    q = _rand(2, Hq, D, seed=702)
    rseq = torch.arange(2, dtype=torch.int32, device=DEV)
    for rctx, max_ctx in (([40, 64 + 16], 4096), ([40, 600], 64)):
        ops.paged_attention(q, kc, vc, bt, rseq, torch.tensor(rctx, dtype=torch.int32, device=DEV), Hq, 0.1,
                            max_ctx=max_ctx, impl=impl)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="status 5"):
            ops.check_status()


@pytest.mark.parametrize("H,ctxs", [(16, [1, 64, 65, 300]), (128, [1000, 17]), (40, [129, 2048, 5])])
def test_mla_decode_latent_attention(H, ctxs):
    """Absorbed MLA attention over the paged 576-wide latent cache against the fp32
    statement; a row whose context exceeds its block table reports OM_ERR_BOUNDS."""
    rows = len(ctxs)
    mb = (max(ctxs) + 15) // 16
    nb = rows * mb + 3
    cache = _rand(nb, 16, 576, seed=700)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(1)).to(DEV).int()
    bt = perm[: rows * mb].view(rows, mb).contiguous()
    q = _rand(rows, H, 576, seed=701, std=0.3)
    row_seq = torch.arange(rows, dtype=torch.int32, device=DEV)
    row_ctx = torch.tensor(ctxs, dtype=torch.int32, device=DEV)
    scale = 1.0 / math.sqrt(192)
    got = ops.mla_decode(q, cache, bt, row_seq, row_ctx, max(ctxs), scale)
    torch.cuda.synchronize()
    ops.check_status()
    want = ref.mla_decode(q.float(), cache.float(), bt, row_seq, row_ctx, scale)
    _close(got, want)
    bad = torch.tensor([mb * 16 + 5] + ctxs[1:], dtype=torch.int32, device=DEV)
    ops.mla_decode(q, cache, bt, row_seq, bad, mb * 16 + 5, scale)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError):
        ops.check_status()


def test_mla_layer_gpu_matches_fp32():
    from openmini_v1_b200.models.config import MLAConfig, tiny
    from openmini_v1_b200.models.llama import DecoderLM, ForwardBatch
    from openmini_v1_b200.models.mla import mla_attention, mla_reference_layer
    cfg = tiny()
    cfg.dtype = "bfloat16"
    cfg.mla = MLAConfig(enabled=True, qk_nope_dim=128, qk_rope_dim=64, v_head_dim=128)
    m = DecoderLM(cfg, device=DEV, seed=1)
    T = 70
    i32 = dict(dtype=torch.int32, device=DEV)
    fb = ForwardBatch(torch.arange(T, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                      torch.arange(5, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                      torch.tensor([T - 1], device=DEV))
    kv = m.allocate_kv(5)
    a = _rand(T, cfg.hidden_size, seed=702)
    got = mla_attention(m, 0, m.layers[0], a, fb, kv)
    torch.cuda.synchronize()
    ops.check_status()
    want = mla_reference_layer(m, m.layers[0], a, fb.positions)
    _close(got, want, rtol=3e-2, atol=3e-2)


def test_dsa_index_scores_tensor_core():
    """Prefill indexer scores through the tcgen05 GEMM + head reduction against the fp32
    statement: two sequence segments, one with a cached prefix (positions 300..449)."""
    from types import SimpleNamespace
    from openmini_v1_b200.models import dsa
    H = 4
    segs = [(0, 300, 150), (1, 0, 100)]  # (sequence, first position, rows)
    rseq = torch.tensor([s for s, p, n in segs for _ in range(n)], dtype=torch.int32, device=DEV)
    rctx = torch.tensor([p + i + 1 for s, p, n in segs for i in range(n)], dtype=torch.int32, device=DEV)
    T = rseq.numel()
    nb = 64
    icache = _rand(nb, 16, 64, seed=80)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(2)).int().to(DEV)
    bt = torch.stack([perm[:32], perm[32:]]).contiguous()
    qi = _rand(T, H * 64, seed=81)
    wi = torch.rand(T, H, device=DEV)
    L = 450
    scores = torch.empty(T, L, device=DEV)
    fb = SimpleNamespace(row_seq=rseq, row_ctx=rctx, block_tables=bt)
    dsa.index_scores_tc(qi, wi, icache, fb, H, scores)
    torch.cuda.synchronize()
    ops.check_status()
    sref = dsa.index_scores_ref(qi.cpu(), wi.cpu(), icache.cpu(), bt.cpu(), rseq.cpu(), rctx.cpu(), H, L)
    fin = torch.isfinite(sref)
    assert torch.equal(torch.isfinite(scores.cpu()), fin)
    err = (scores.cpu()[fin] - sref[fin]).abs()
    assert float(err.max()) < 2e-2 * float(sref[fin].abs().max())


@pytest.mark.parametrize("typ", [2, 8, 12, 13, 14])
def test_gguf_device_dequant(typ):
    """GGUF blocks expanded on the GPU equal the host readers (bf16 rounding of the result)."""
    import numpy as np
    from openmini_v1_b200.gguf.constants import BLOCK_SIZES, GGMLType
    from openmini_v1_b200.gguf.device import dequantize_to_device
    from openmini_v1_b200.gguf.quants import dequantize
    per, nbytes = BLOCK_SIZES[GGMLType(typ)]
    nblk = 64
    rng = np.random.default_rng(typ)
    b = rng.integers(0, 256, size=(nblk, nbytes), dtype=np.uint8)
    f16_at = {2: (0,), 8: (0,), 12: (0, 2), 13: (0, 2), 14: (208,)}[typ]
    for off in f16_at:
        b[:, off:off + 2] = np.frombuffer(rng.uniform(-0.1, 0.1, nblk).astype(np.float16).tobytes(),
                                          np.uint8).reshape(nblk, 2)
    want = torch.from_numpy(dequantize(b.reshape(-1), typ, nblk * per)).view(4, -1)
    got = dequantize_to_device(b.reshape(-1), typ, (4, nblk * per // 4), DEV)
    # fp32 products on both sides; a fused multiply-add may move the bf16 rounding by one step
    torch.testing.assert_close(got.float().cpu(), want.to(torch.bfloat16).float(), rtol=8e-3, atol=1e-6)


def test_tts_acoustic_model_gpu():
    """TTS acoustic model on the GPU kernels (GEMM, LayerNorm, GELU, bidirectional
    FlashAttention at head_dim 128) against the same model's fp32 CPU statement with the
    GPU's durations (rounding of a duration near .5 may differ between precisions);
    the vocoder output is finite and as long as the durations say."""
    from openmini_v1_b200.models.tts import TTSModel
    g = TTSModel(device=DEV, seed=5)
    c = TTSModel(device="cpu", dtype=torch.float32, seed=5)
    text = "the quick brown fox"
    _, d = g.durations(text, "v", 1.0)
    got = g.mel(text, "v", 1.0, d=d)
    ops.check_status()
    _close(got.cpu(), c.mel(text, "v", 1.0, d=d.cpu()), rtol=5e-2, atol=5e-2)
    wav = g.vocode(got)
    assert torch.isfinite(wav).all() and wav.numel() == (int(d.sum()) - 1) * g.cfg.hop
