"""Per-kernel microbenchmark of the sm_100a hot ops, with roofline fractions.

    python -m openmini_v1_b200.ops.microbench --op gemm_q4 --m 32 --n 10240 --k 8192
    python -m openmini_v1_b200.ops.microbench --op all

Each case is timed with CUDA events on the launching stream after warm-up, one
launch per timed interval, with a 256 MiB write between intervals so that every
launch starts with a cold L2 (126 MB on B200). ``--iters`` sets how many
launches are timed (the median is reported); for an ncu capture use a small
``--iters``/``--warmup`` and ``-k``/``-c`` on the ncu side.

The achieved bandwidth / FLOP rate is divided by the measured copy bandwidth and
cuBLAS bf16 rate in ``MEASURED_PEAKS.json`` at the repository root (driver
written) or, if absent, by 6650 GB/s and 1590 TFLOP/s.

Bytes are the algorithmic minimum: every operand read once, every output
written once (packed 4-bit weights at 0.5 B + one bf16 scale per 32 values).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics

import torch

from .. import ops

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(_ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def _time(fn, iters, warmup):
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.fill_(1.0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ops.check_status()
    return statistics.median(ts)


def _rand(*shape, dtype=torch.bfloat16, std=1.0):
    return (torch.randn(*shape, device="cuda") * std).to(dtype)


def case_gemm(m, n, k, kind):
    from ..models.quantize import Int8Weight, Q4Weight
    x = _rand(m, k)
    w = _rand(n, k, std=0.02)
    if kind == "bf16":
        wb = w
        wbytes = n * k * 2
    elif kind == "q4":
        wb = Q4Weight.from_dense(w)
        wbytes = n * k // 2 + n * (k // 32) * 2
    else:
        wb = Int8Weight.from_dense(w)
        wbytes = n * k + n * 2
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    fn = lambda: ops.linear(x, wb, out=out)  # noqa: E731
    return fn, wbytes + m * k * 2 + m * n * 2, 2.0 * m * n * k


def _paged(S, Hkv, D, lens):
    nb = sum((l + 15) // 16 for l in lens) + 4
    kc = _rand(nb, Hkv, 16, D)
    vc = _rand(nb, Hkv, 16, D)
    mb = max((l + 15) // 16 for l in lens)
    perm = torch.randperm(nb, device="cuda").to(torch.int32)
    bt = torch.zeros(S, mb, dtype=torch.int32, device="cuda")
    o = 0
    for s, l in enumerate(lens):
        c = (l + 15) // 16
        bt[s, :c] = perm[o:o + c]
        o += c
    return kc, vc, bt


def case_decode_attn(batch, ctx, hq, hkv, d=128, impl="tc"):
    lens = [ctx] * batch
    kc, vc, bt = _paged(batch, hkv, d, lens)
    q = _rand(batch, hq, d)
    rseq = torch.arange(batch, dtype=torch.int32, device="cuda")
    rctx = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = torch.empty(batch, hq * d, dtype=torch.bfloat16, device="cuda")
    sc = 1 / math.sqrt(d)
    fn = lambda: ops.paged_attention(q, kc, vc, bt, rseq, rctx, hq, sc, max_ctx=ctx, out=out, impl=impl)  # noqa
    kv_bytes = 2 * batch * ctx * hkv * d * 2
    return fn, kv_bytes + 2 * q.numel() * 2, 4.0 * batch * ctx * hq * d


def case_prefill_attn(seqs, seqlen, hq, hkv, d=128):
    from ..engine.engine import LLMEngine
    lens = [seqlen] * seqs
    kc, vc, bt = _paged(seqs, hkv, d, lens)
    T = seqs * seqlen
    qkv = _rand(T, (hq + 2 * hkv) * d)
    rseq = torch.arange(seqs, dtype=torch.int32, device="cuda").repeat_interleave(seqlen)
    rctx = torch.arange(1, seqlen + 1, dtype=torch.int32, device="cuda").repeat(seqs)

    class _C:
        def __init__(self, n):
            self.start, self.end = 0, n

    class _SO:
        kind = "prefill"

    tiles = torch.tensor(LLMEngine._prefill_tiles(_SO, [_C(seqlen) for _ in range(seqs)], T), dtype=torch.int32,
                         device="cuda")
    out = torch.empty(T, hq * d, dtype=torch.bfloat16, device="cuda")
    sc = 1 / math.sqrt(d)
    fn = lambda: ops.flash_prefill(qkv, kc, vc, bt, rseq, rctx, tiles, hq, sc, out=out)  # noqa: E731
    flops = 4.0 * seqs * hq * d * seqlen * (seqlen + 1) / 2  # causal
    return fn, qkv.numel() * 2 + out.numel() * 2 + 2 * T * hkv * d * 2, flops


def case_rmsnorm(rows, dim):
    x = _rand(rows, dim)
    dlt = _rand(rows, dim)
    w = _rand(dim)
    out = torch.empty_like(x)
    fn = lambda: ops.rmsnorm(x, w, 1e-5, out=out, delta=dlt)  # noqa: E731
    return fn, 4 * rows * dim * 2, 0.0


def case_sample(batch, vocab):
    lg = _rand(batch, vocab, dtype=torch.float32)
    t = torch.full((batch,), 0.7, device="cuda")
    p = torch.full((batch,), 0.9, device="cuda")
    k = torch.zeros(batch, dtype=torch.int32, device="cuda")
    rng = torch.randint(0, 1 << 40, (batch, 2), device="cuda")
    fn = lambda: ops.sample(lg, t, p, k, rng, want_mask=True)  # noqa: E731
    return fn, lg.numel() * 4, 0.0


# name -> (builder, kwargs); the "all" sweep. Shapes are those of the 70B-shape decoder.
def case_mla_decode(batch, ctx, heads):
    """Absorbed MLA decode over a paged 576-wide latent cache (csrc/attn/mla.cu)."""
    nb = batch * ((ctx + 15) // 16) + 4
    cache = _rand(nb, 16, 576)
    perm = torch.randperm(nb, device="cuda").to(torch.int32)
    mb = (ctx + 15) // 16
    bt = perm[: batch * mb].view(batch, mb).contiguous()
    q = _rand(batch, heads, 576)
    rseq = torch.arange(batch, dtype=torch.int32, device="cuda")
    rctx = torch.full((batch,), ctx, dtype=torch.int32, device="cuda")
    out = torch.empty(batch, heads, 512, dtype=torch.bfloat16, device="cuda")
    fn = lambda: ops.mla_decode(q, cache, bt, rseq, rctx, ctx, 1 / math.sqrt(192), out=out)  # noqa
    return fn, batch * ctx * 576 * 2 + q.numel() * 2 + out.numel() * 2, 2.0 * batch * heads * ctx * (576 + 512)


def case_dsa_index_tc(rows, keys, heads=4):
    """DSA prefill indexer scores on tensor cores: one sequence, rows ending at position keys."""
    from types import SimpleNamespace
    from ..models.dsa import index_scores_tc
    nb = (keys + 15) // 16 + 2
    icache = _rand(nb, 16, 64)
    bt = torch.randperm(nb, device="cuda").to(torch.int32)[None, : (keys + 15) // 16].contiguous()
    qi = _rand(rows, heads * 64)
    wi = torch.rand(rows, heads, device="cuda")
    fb = SimpleNamespace(row_seq=torch.zeros(rows, dtype=torch.int32, device="cuda"),
                         row_ctx=torch.arange(keys - rows + 1, keys + 1, dtype=torch.int32, device="cuda"),
                         block_tables=bt)
    scores = torch.empty(rows, keys, device="cuda")
    fn = lambda: index_scores_tc(qi, wi, icache, fb, heads, scores)  # noqa
    return fn, rows * keys * 4 + keys * 128, 2.0 * rows * heads * keys * 64


def case_dsa_sparse_decode(batch, ctx, hq, hkv, k=2048, d=128):
    """DSA sparse attention at decode: each row attends to k selected keys of its
    ctx-token paged KV (split over CTAs when rows x KV heads would not fill the GPU)."""
    from .. import _native
    mb = ctx // 16
    nb = batch * mb
    kc, vc = _rand(nb, hkv, 16, d, std=0.5), _rand(nb, hkv, 16, d)
    bt = torch.randperm(nb, device="cuda").to(torch.int32).view(batch, mb).contiguous()
    rseq = torch.arange(batch, dtype=torch.int32, device="cuda")
    sel = torch.stack([torch.randperm(ctx, device="cuda")[:k] for _ in range(batch)]).to(torch.int32)
    n = torch.full((batch,), k, dtype=torch.int32, device="cuda")
    q = _rand(batch, hq * d)
    out = torch.empty(batch, hq * d, dtype=torch.bfloat16, device="cuda")
    fn = lambda: _native.C().dsa_attention(q, kc, vc, bt, rseq, sel, n, out, hq, 1 / math.sqrt(d))  # noqa
    return fn, batch * k * hkv * d * 2 * 2 + q.numel() * 4, 4.0 * batch * hq * k * d


SUITE = {
    "gemm_bf16_decode_qkv": (case_gemm, dict(m=32, n=10240, k=8192, kind="bf16")),
    "gemm_q4_decode_qkv": (case_gemm, dict(m=32, n=10240, k=8192, kind="q4")),
    "gemm_q4_decode_gateup": (case_gemm, dict(m=32, n=57344, k=8192, kind="q4")),
    "gemm_q4_decode_down": (case_gemm, dict(m=32, n=8192, k=28672, kind="q4")),
    "gemm_i8_decode_qkv": (case_gemm, dict(m=32, n=10240, k=8192, kind="int8")),
    "gemm_i8_decode_gateup": (case_gemm, dict(m=32, n=57344, k=8192, kind="int8")),
    # per-GPU gate/up shapes under TP 2 / 4 / 8 with 32 requests per GPU (weak scaling)
    "gemm_q4_decode_gateup_tp2": (case_gemm, dict(m=64, n=28672, k=8192, kind="q4")),
    "gemm_q4_decode_gateup_tp4": (case_gemm, dict(m=128, n=14336, k=8192, kind="q4")),
    "gemm_q4_decode_gateup_tp8": (case_gemm, dict(m=256, n=7168, k=8192, kind="q4")),
    "gemm_bf16_prefill": (case_gemm, dict(m=4096, n=8192, k=8192, kind="bf16")),
    "gemm_q4_prefill": (case_gemm, dict(m=4096, n=8192, k=8192, kind="q4")),
    "attn_decode_tc": (case_decode_attn, dict(batch=32, ctx=4096, hq=64, hkv=8)),
    "attn_prefill_tc": (case_prefill_attn, dict(seqs=4, seqlen=4096, hq=64, hkv=8)),
    "rmsnorm_residual": (case_rmsnorm, dict(rows=16384, dim=8192)),
    "sampler_topp_mask": (case_sample, dict(batch=256, vocab=128256)),
    "mla_decode": (case_mla_decode, dict(batch=32, ctx=4096, heads=128)),
    "dsa_index_tc_prefill": (case_dsa_index_tc, dict(rows=4096, keys=32768)),
    "dsa_sparse_decode": (case_dsa_sparse_decode, dict(batch=2, ctx=32768, hq=40, hkv=8)),
}


def run(name, builder, kw, iters, warmup):
    hbm, tf, src = peaks()
    fn, nbytes, flops = builder(**kw)
    ms = _time(fn, iters, warmup)
    gbs = nbytes / ms / 1e6
    tfl = flops / ms / 1e9
    res = {"case": name, **kw, "ms": round(ms, 4), "GB/s": round(gbs, 1), "TFLOP/s": round(tfl, 1),
           f"hbm_frac_of_{src}": round(gbs / hbm, 3), f"tc_frac_of_{src}": round(tfl / tf, 3)}
    print(json.dumps(res), flush=True)
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="all", help="a SUITE name, 'all', or gemm_bf16/gemm_q4/gemm_int8/attn_decode/"
                                                "attn_prefill/rmsnorm/sample with the shape flags")
    ap.add_argument("--m", type=int, default=32)
    ap.add_argument("--n", type=int, default=10240)
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--hq", type=int, default=64)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args(argv)
    torch.manual_seed(0)
    if a.op == "all":
        for name, (b, kw) in SUITE.items():
            run(name, b, kw, a.iters, a.warmup)
        return
    if a.op in SUITE:
        b, kw = SUITE[a.op]
        run(a.op, b, kw, a.iters, a.warmup)
        return
    table = {
        "gemm_bf16": (case_gemm, dict(m=a.m, n=a.n, k=a.k, kind="bf16")),
        "gemm_q4": (case_gemm, dict(m=a.m, n=a.n, k=a.k, kind="q4")),
        "gemm_int8": (case_gemm, dict(m=a.m, n=a.n, k=a.k, kind="int8")),
        "attn_decode": (case_decode_attn, dict(batch=a.batch, ctx=a.ctx, hq=a.hq, hkv=a.hkv)),
        "attn_prefill": (case_prefill_attn, dict(seqs=a.batch, seqlen=a.ctx, hq=a.hq, hkv=a.hkv)),
        "rmsnorm": (case_rmsnorm, dict(rows=a.m, dim=a.k)),
        "sample": (case_sample, dict(batch=a.batch, vocab=a.n)),
    }
    b, kw = table[a.op]
    run(a.op, b, kw, a.iters, a.warmup)


if __name__ == "__main__":
    main()
