"""Dynamic Sparse Attention layer (14B long-context configuration).

Per layer a lightweight indexer projects the normed hidden state to H_I query
heads of 64 dims, one 64-dim key and H_I head weights:

    I(t, s) = sum_h w_h(t) * relu(q_h(t) . k(s))

Indexer keys live in their own paged cache (``KVCache.idx_k``, one 64-dim row
per token, same block table as K/V). When a row's context reaches
``dsa.threshold`` it attends only to its top-k scoring keys (k = dsa.top_k,
or the reference's dynamic k of 512 / 1024 / 2048 / 4096 for contexts up to
1K / 4K / 8K / beyond, openmini-server/src/model/inference/dsa.rs:244-297);
shorter contexts use dense paged attention. Under tensor parallelism every
rank scores with the same (replicated) indexer and attends with its own KV
heads.
"""
from __future__ import annotations

import torch

from .. import _native, ops
from ..ops import reference as ref


def dynamic_k(ctx: int, base: int = 2048) -> int:
    if ctx <= 1024:
        return 512
    if ctx <= 4096:
        return 1024
    if ctx <= 8192:
        return 2048
    return 4096


def init_indexer(model, gen, std):
    d = model.cfg.dsa
    D = model.cfg.hidden_size
    rows = d.indexer_heads * d.indexer_dim + d.indexer_dim + d.indexer_heads
    return {"indexer": model._randn(gen, rows, D, std=std)}


def _split(model, proj):
    d = model.cfg.dsa
    H, Di = d.indexer_heads, d.indexer_dim
    qi = proj[:, :H * Di]
    ki = proj[:, H * Di:H * Di + Di]
    wi = proj[:, H * Di + Di:H * Di + Di + H].float()
    return qi, ki, wi


def index_scores_ref(qi, wi, icache, block_tables, row_seq, row_ctx, H, s_ld):
    rows = row_seq.shape[0]
    out = torch.full((rows, s_ld), float("-inf"))
    for r in range(rows):
        n = int(row_ctx[r])
        bt = block_tables[int(row_seq[r])]
        idx = torch.arange(n)
        K = icache[bt[(idx // 16).long()].long(), idx % 16].float()     # [n, 64]
        q = qi[r].float().view(H, -1)                                   # [H, 64]
        out[r, :n] = (torch.relu(q @ K.t()) * wi[r].float()[:, None]).sum(0)
    return out


def topk_ref(scores, row_ctx, k):
    rows = scores.shape[0]
    idx = torch.full((rows, k), -1, dtype=torch.int32)
    n = torch.zeros(rows, dtype=torch.int32)
    for r in range(rows):
        c = int(row_ctx[r])
        kk = min(k, c)
        s = scores[r, :c].float()
        if kk < c:
            thr = torch.topk(s, kk).values[-1]
            gt = torch.nonzero(s > thr).flatten()
            eq = torch.nonzero(s == thr).flatten()[: kk - gt.numel()]
            sel = torch.cat([gt, eq])
        else:
            sel = torch.arange(c)
        idx[r, :kk] = sel.to(torch.int32)
        n[r] = kk
    return idx, n


def sparse_attention_ref(q, k_cache, v_cache, block_tables, row_seq, sel, sel_n, Hq, scale):
    rows = row_seq.shape[0]
    Hkv, D = k_cache.shape[1], k_cache.shape[3]
    G = Hq // Hkv
    out = torch.empty(rows, Hq * D, dtype=q.dtype)
    qv = q.reshape(rows, -1)[:, :Hq * D].reshape(rows, Hq, D).float()
    for r in range(rows):
        keys = sel[r, :int(sel_n[r])].long()
        bt = block_tables[int(row_seq[r])]
        blk = bt[(keys // 16).long()].long()
        K = k_cache[blk, :, keys % 16].float().repeat_interleave(G, 1)
        V = v_cache[blk, :, keys % 16].float().repeat_interleave(G, 1)
        p = torch.softmax(torch.einsum("hd,nhd->hn", qv[r], K) * scale, -1)
        out[r] = torch.einsum("hn,nhd->hd", p, V).reshape(-1).to(q.dtype)
    return out


def dsa_attention(model, i, L, a, qkv, fb, kv):
    cfg = model.cfg
    d = cfg.dsa
    T = a.shape[0]
    proj = ops.linear(a, L["indexer"])
    qi, ki, wi = _split(model, proj)
    _write_index(ki, fb.slots, kv.idx_k[i])
    if fb.max_ctx < d.threshold:
        return ops.paged_attention(qkv, kv.k[i], kv.v[i], fb.block_tables, fb.row_seq, fb.row_ctx, model.hq,
                                   model.scale, fb.max_ctx)
    k = d.top_k
    s_ld = fb.max_ctx
    if a.is_cuda:
        c = ops.ctx(a.device)
        scores = c.workspace("dsa_scores", T * s_ld)[:T * s_ld].view(T, s_ld)
        if T >= TC_MIN_ROWS:
            index_scores_tc(qi, wi.contiguous(), kv.idx_k[i], fb, d.indexer_heads, scores)
        else:
            _native.C().dsa_scores(qi, wi.contiguous(), d.indexer_heads, kv.idx_k[i], fb.block_tables, fb.row_seq,
                                   fb.row_ctx, scores, c.status)
        sel = torch.empty(T, k, dtype=torch.int32, device=a.device)
        n = torch.empty(T, dtype=torch.int32, device=a.device)
        _native.C().dsa_topk(scores, fb.row_ctx, k, sel, n)
        out = torch.empty(T, model.hq * model.hd, dtype=qkv.dtype, device=a.device)
        _native.C().dsa_attention(qkv, kv.k[i], kv.v[i], fb.block_tables, fb.row_seq, sel, n, out, model.hq,
                                  model.scale)
        return out
    scores = index_scores_ref(qi, wi, kv.idx_k[i], fb.block_tables, fb.row_seq, fb.row_ctx, d.indexer_heads, s_ld)
    sel, n = topk_ref(scores, fb.row_ctx, k)
    return sparse_attention_ref(qkv, kv.k[i], kv.v[i], fb.block_tables, fb.row_seq, sel, n, model.hq, model.scale)


TC_MIN_ROWS = 64          # prefill batches score on tensor cores; decode rows keep the bandwidth-bound kernel
TC_MAX_GEMM_BYTES = 256 << 20


def index_scores_tc(qi, wi, icache, fb, H: int, scores):
    """Indexer scores of a prefill batch on tensor cores: per sequence segment of the
    batch, its indexer keys are gathered contiguously ([S, 64], S rounded up to 64), the
    tcgen05 GEMM computes every (row, head) dot product (q rows [n H, 64] x keys^T), and
    ``dsa_head_reduce`` applies ReLU, the head weights and the causal mask into the
    fp32 score rows. Rows are processed in chunks whose GEMM output stays under
    ``TC_MAX_GEMM_BYTES``."""
    Di = icache.shape[-1]
    seq = fb.row_seq.cpu().tolist()
    ctx = fb.row_ctx.cpu().tolist()
    flat = icache.view(-1, Di)
    T = len(seq)
    r0 = 0
    while r0 < T:
        r1 = r0
        while r1 < T and seq[r1] == seq[r0]:
            r1 += 1
        S = max(ctx[r0:r1])
        Sp = (S + 63) // 64 * 64
        pos = torch.arange(Sp, device=qi.device)
        blk = fb.block_tables[seq[r0]].long()[(pos // 16).clamp(max=fb.block_tables.shape[1] - 1)]
        keys = flat[(blk.clamp(min=0) * 16 + pos % 16).clamp(max=flat.shape[0] - 1)].contiguous()
        step = max(1, TC_MAX_GEMM_BYTES // (H * Sp * 2))
        for c0 in range(r0, r1, step):
            c1 = min(r1, c0 + step)
            q = qi[c0:c1].reshape((c1 - c0) * H, Di).contiguous()
            g = ops.linear(q, keys)  # [rows * H, Sp] on the tcgen05 GEMM
            _native.C().dsa_head_reduce(g, S, wi[c0:c1], H, fb.row_ctx[c0:c1], scores[c0:c1])
        r0 = r1


def _write_index(ki, slots, icache):
    """Store one 64-dim indexer key per token at its cache slot (slot < 0: skip)."""
    flat = icache.view(-1, icache.shape[-1])
    s = slots.long().clamp(min=0)
    keep = (slots >= 0)[:, None]
    flat[s] = torch.where(keep, ki.to(icache.dtype), flat[s])  # no host sync (graph-safe)
