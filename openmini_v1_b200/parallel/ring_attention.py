"""Context parallelism: ring attention over a sequence split across ranks.

Rank r of W holds the queries and keys/values of tokens [r C, (r+1) C). The KV
chunks travel around the ring (rank r sends to r+1 and receives from r-1 with
asynchronous point-to-point ops, so the next chunk is in flight while the
current one is attended). At step s rank r holds the chunk of rank r - s; it
attends to it causally at s = 0 (its own chunk) and fully for earlier chunks,
and skips chunks from later positions. Partial results are combined with their
log-sum-exp: o = sum_i exp(lse_i - lse) o_i, lse = log sum_i exp(lse_i).

On the GPU each partial runs the tcgen05 FlashAttention kernel, which also
writes the per-row log-sum-exp; the received chunk is laid out as a paged cache
(16-token blocks) for it. On CPU the same steps run as fp32 math (tests).

Reference counterpart: the "ring" path of the reference's ring/flash/linear
hybrid (openmini-server/src/model/inference/ring_flash_linear.rs:538-700), which
is block-local attention inside one process with no KV rotation.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


def _attend_cpu(q, k, v, scale, causal):
    """q [Tq, H, D], k/v [Tk, Hkv, D] -> (out fp32 [Tq, H, D], lse fp32 [Tq, H])."""
    H, Hkv = q.shape[1], k.shape[1]
    g = H // Hkv
    kf = k.float().repeat_interleave(g, dim=1)
    vf = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kf) * scale
    if causal:
        Tq, Tk = q.shape[0], k.shape[0]
        mask = torch.arange(Tk)[None, :] > torch.arange(Tq)[:, None] + (Tk - Tq)
        s = s.masked_fill(mask[None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)                       # [H, Tq]
    p = torch.exp(s - lse[..., None])
    out = torch.einsum("hqk,khd->qhd", p, vf)
    return out, lse.transpose(0, 1).contiguous()


def _attend_cuda(q, k, v, scale, causal):
    from .. import ops
    Tq, H, D = q.shape
    Tk, Hkv = k.shape[0], k.shape[1]
    nb = (Tk + 15) // 16
    pad = nb * 16 - Tk

    def paged(x):
        if pad:
            x = torch.cat([x, x.new_zeros(pad, Hkv, D)])
        return x.view(nb, 16, Hkv, D).transpose(1, 2).contiguous()  # [blocks, Hkv, 16, D]

    kc, vc = paged(k), paged(v)
    dev = q.device
    bt = torch.arange(nb, dtype=torch.int32, device=dev)[None]
    if causal:
        row_ctx = torch.arange(Tk - Tq + 1, Tk + 1, dtype=torch.int32, device=dev)
    else:
        row_ctx = torch.full((Tq,), Tk, dtype=torch.int32, device=dev)
    tiles = []
    for t0 in range(0, Tq, 128):
        rows = min(128, Tq - t0)
        tiles.append((t0, rows, 0, int(Tk - Tq + t0 + rows) if causal else Tk))
    tiles.sort(key=lambda x: -x[3])
    tiles = torch.tensor(tiles, dtype=torch.int32, device=dev)
    out = torch.empty(Tq, H * D, dtype=q.dtype, device=dev)
    lse = torch.empty(Tq, H, dtype=torch.float32, device=dev)
    rseq = torch.zeros(Tq, dtype=torch.int32, device=dev)
    ops.flash_prefill(q.reshape(Tq, H * D).contiguous(), kc, vc, bt, rseq, row_ctx, tiles, H, scale, out=out,
                      lse=lse)
    return out.view(Tq, H, D).float(), lse


def attend(q, k, v, scale, causal):
    if q.is_cuda:
        return _attend_cuda(q, k, v, scale, causal)
    return _attend_cpu(q, k, v, scale, causal)


def merge(o_a, lse_a, o_b, lse_b):
    """Combine two attention partials over disjoint key sets."""
    m = torch.maximum(lse_a, lse_b)
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    wa, wb = torch.exp(lse_a - m), torch.exp(lse_b - m)
    den = wa + wb
    o = (o_a * wa[..., None] + o_b * wb[..., None]) / den.clamp_min(1e-30)[..., None]
    return o, m + torch.log(den)


def ring_attention(q, k, v, scale: float | None = None, group=None):
    """Causal attention of this rank's query chunk over the whole sequence.

    q [C, H, D], k / v [C, Hkv, D]: this rank's contiguous chunk (all ranks equal C).
    Returns (out [C, H, D] in q's dtype, lse [C, H] fp32)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    W = dist.get_world_size(group) if dist.is_initialized() else 1
    r = dist.get_rank(group) if dist.is_initialized() else 0
    if W == 1:
        out, lse = attend(q, k, v, scale, causal=True)
        return out.to(q.dtype), lse
    g = (lambda i: dist.get_global_rank(group, i)) if group is not None else (lambda i: i)
    nxt, prv = g((r + 1) % W), g((r - 1) % W)
    cur = torch.stack([k, v]).contiguous()
    out = lse = None
    for step in range(W):
        works, recv = None, None
        if step < W - 1:  # the next chunk is in flight while this one is attended
            recv = torch.empty_like(cur)
            works = dist.batch_isend_irecv([dist.P2POp(dist.isend, cur, nxt, group),
                                            dist.P2POp(dist.irecv, recv, prv, group)])
        src = (r - step) % W
        if step == 0:
            out, lse = attend(q, cur[0], cur[1], scale, causal=True)
        elif src < r:  # an earlier chunk: fully visible
            o_s, l_s = attend(q, cur[0], cur[1], scale, causal=False)
            out, lse = merge(out, lse, o_s, l_s)
        if works is not None:
            for w in works:
                w.wait()
            cur = recv
    return out.to(q.dtype), lse
