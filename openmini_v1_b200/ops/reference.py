"""Plain PyTorch fp32 statements of every kernel in ``csrc/``.

These are (1) the numerics oracle the GPU tests compare against and (2) the
CPU execution path used by the plumbing configuration (tiny model on CPU).
Semantics match the kernels, including cache layouts, rounding points that
matter (the residual is rounded to the activation dtype before it is
normalised), quantiser rounding and the sampler's Philox stream.
"""
from __future__ import annotations

import math

import numpy as np
import torch

BLOCK = 16


def linear(x, w, resid=None):
    y = x.float() @ w.float().t()
    if resid is not None:
        y = y + resid.float()
    return y.to(x.dtype)


def rmsnorm(x, w, eps, delta=None):
    """out = x / rms(x) * w; with ``delta`` x is first updated in place to x + delta."""
    if delta is not None:
        x.copy_((x.float() + delta.float()).to(x.dtype))
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * inv * w.float()).to(x.dtype)


def layernorm(x, w, b, eps):
    xf = x.float()
    mu = xf.mean(-1, keepdim=True)
    var = (xf - mu).pow(2).mean(-1, keepdim=True)
    y = (xf - mu) * torch.rsqrt(var + eps) * w.float()
    if b is not None:
        y = y + b.float()
    return y.to(x.dtype)


def silu_mul(gu):
    F = gu.shape[-1] // 2
    g, u = gu[..., :F].float(), gu[..., F:].float()
    return (g / (1 + torch.exp(-g)) * u).to(gu.dtype)


def gelu(x):
    xf = x.float()
    return (0.5 * xf * (1 + torch.tanh(0.7978845608028654 * (xf + 0.044715 * xf ** 3)))).to(x.dtype)


def softmax(x, scale=1.0):
    return torch.softmax(x.float() * scale, dim=-1)


def inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    i = torch.arange(0, head_dim // 2, dtype=torch.float64)
    return (1.0 / (theta ** (2 * i / head_dim))).float()


def rope(x, positions, inv_f, mode=0):
    """Rotate [T, H, D] by position. mode 0 = interleaved pairs, 1 = half split."""
    T, H, D = x.shape
    ang = positions.double()[:, None] * inv_f.double().to(positions.device)[None, :]  # [T, D/2]
    c, s = torch.cos(ang).float()[:, None, :], torch.sin(ang).float()[:, None, :]
    xf = x.float()
    if mode == 0:
        x0, x1 = xf[..., 0::2], xf[..., 1::2]
        out = torch.empty_like(xf)
        out[..., 0::2] = x0 * c - x1 * s
        out[..., 1::2] = x0 * s + x1 * c
    else:
        h = D // 2
        x0, x1 = xf[..., :h], xf[..., h:]
        out = torch.cat([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1)
    return out.to(x.dtype)


def rope_kv(qkv, positions, slots, k_cache, v_cache, inv_f, Hq, Hkv, D, mode=0):
    """In-place RoPE on the q and k parts of qkv rows and write k, v into the paged cache."""
    T = qkv.shape[0]
    if T == 0:
        return
    q = qkv[:, : Hq * D].view(T, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D:(Hq + 2 * Hkv) * D].view(T, Hkv, D)
    q.copy_(rope(q, positions, inv_f, mode))
    k.copy_(rope(k, positions, inv_f, mode))
    kv_write(k, v, slots, k_cache, v_cache)


def kv_write(k, v, slots, k_cache, v_cache):
    m = slots >= 0
    s = slots[m].long()
    blk, off = s // BLOCK, s % BLOCK
    k_cache[blk, :, off, :] = k[m].to(k_cache.dtype)
    v_cache[blk, :, off, :] = v[m].to(v_cache.dtype)


def gather_kv(cache, block_table, n):
    """[n, Hkv, D] keys of one sequence from a paged cache [blocks, Hkv, 16, D]."""
    idx = torch.arange(n, device=cache.device)
    blk = block_table[(idx // BLOCK).long()].long()
    return cache[blk, :, idx % BLOCK, :]


def paged_attention(q, k_cache, v_cache, block_tables, row_seq, row_ctx, Hq, scale):
    """q [rows, Hq, D] (or [rows, >=Hq*D]); row r attends to the first row_ctx[r] keys of its sequence."""
    rows = row_seq.shape[0]
    Hkv, D = k_cache.shape[1], k_cache.shape[3]
    G = Hq // Hkv
    out = torch.empty(rows, Hq, D, dtype=q.dtype, device=q.device)
    qv = q.reshape(rows, -1)[:, : Hq * D].reshape(rows, Hq, D).float()
    for r in range(rows):
        n = int(row_ctx[r])
        bt = block_tables[int(row_seq[r])]
        K = gather_kv(k_cache, bt, n).float().repeat_interleave(G, dim=1)  # [n, Hq, D]
        V = gather_kv(v_cache, bt, n).float().repeat_interleave(G, dim=1)
        s = torch.einsum("hd,nhd->hn", qv[r], K) * scale
        p = torch.softmax(s, dim=-1)
        out[r] = torch.einsum("hn,nhd->hd", p, V).to(q.dtype)
    return out


def embedding(ids, table):
    return table[ids.long()]


# ------------------------------------------------------------------ weight quantisation
def quantize_q4(w):
    """bf16 [N, K] -> (uint8 [N, K/2], bf16 scales [N, K/32]); ggml Q4_0 quantiser,
    scale rounded fp16 then bf16, byte i = element i | element i+16 << 4 per block."""
    N, K = w.shape
    b = w.float().reshape(N, K // 32, 32)
    idx = b.abs().argmax(-1, keepdim=True)
    mx = b.gather(-1, idx).squeeze(-1)
    d = (mx / -8.0).half().float().bfloat16().float()
    inv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    q = torch.floor(b * inv[..., None] + 8.5).clamp(0, 15).to(torch.uint8)
    packed = q[..., :16] | (q[..., 16:] << 4)
    return packed.reshape(N, K // 2).contiguous(), d.bfloat16()


def dequant_q4(q, scales):
    N = q.shape[0]
    K = q.shape[1] * 2
    b = q.reshape(N, K // 32, 16)
    lo = (b & 15).float() - 8
    hi = (b >> 4).float() - 8
    v = torch.cat([lo, hi], dim=-1) * scales.float().reshape(N, K // 32, 1)
    return v.reshape(N, K).bfloat16()


def quantize_int8(w):
    wf = w.float()
    s = (wf.abs().amax(-1) / 127.0).half().float()
    inv = torch.where(s > 0, 1.0 / s, torch.zeros_like(s))
    q = torch.round(wf * inv[:, None]).clamp(-127, 127).to(torch.int8)
    return q, s


def dequant_int8(q, s):
    return (q.float() * s[:, None]).bfloat16()


# ------------------------------------------------------------------ sampler
_M0, _M1, _W0, _W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
_MASK = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Philox-4x32-10 (Salmon et al., SC'11) on numpy uint64 arrays holding 32-bit words."""
    c = [np.asarray(x, dtype=np.uint64) & _MASK for x in (c0, c1, c2, c3)]
    k0 = np.uint64(k0) & _MASK
    k1 = np.uint64(k1) & _MASK
    for _ in range(10):
        p0 = np.uint64(_M0) * c[0]
        p1 = np.uint64(_M1) * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
        k0 = (k0 + np.uint64(_W0)) & _MASK
        k1 = (k1 + np.uint64(_W1)) & _MASK
    return c


def _cutoff_mask(x, k, p):
    """Kept set for top-k then top-p over scaled, max-shifted logits x (1-D fp32)."""
    V = x.numel()
    keep = torch.ones(V, dtype=torch.bool, device=x.device)
    if 0 < k < V:
        kth = torch.topk(x, k).values[-1]
        keep &= x >= kth
    if p < 1.0:
        zk = (torch.exp(x) * keep).sum()
        vals = torch.sort(torch.where(keep, x, torch.full_like(x, -math.inf)), descending=True).values
        cs = torch.cumsum(torch.exp(vals), 0)
        idx = int(torch.searchsorted(cs, (p * zk).reshape(1)).clamp(max=V - 1))
        keep &= x >= vals[idx]
    return keep


def sample(logits, temperature, top_p, top_k, rng):
    """Returns (tokens int32 [B], logprob fp32 [B], keep mask bool [B, V]).

    Row b draws with Philox counter (token, 0, offset) under key = its seed: the draw
    depends on the request's (seed, offset) only, not on its position in the batch."""
    B, V = logits.shape
    toks = torch.empty(B, dtype=torch.int32)
    lps = torch.empty(B, dtype=torch.float32)
    masks = torch.zeros(B, V, dtype=torch.bool)
    for b in range(B):
        t = float(temperature[b])
        row = logits[b].float().cpu()
        greedy = not (t > 0)
        xs = row * (1.0 if greedy else 1.0 / t)
        x = xs - xs.max()
        logz = torch.logsumexp(x, 0)
        if greedy:
            keep = x >= 0
            score = x
        else:
            keep = _cutoff_mask(x, int(top_k[b]), float(top_p[b]))
            seed, off = int(rng[b][0]) & 0xFFFFFFFFFFFFFFFF, int(rng[b][1]) & 0xFFFFFFFFFFFFFFFF
            ids = np.arange(V, dtype=np.uint64)
            c = philox4x32_10(ids, np.zeros(V, dtype=np.uint64), np.full(V, off & 0xFFFFFFFF), np.full(V, off >> 32),
                              seed & 0xFFFFFFFF, seed >> 32)
            u = (c[0].astype(np.float64) + 0.5) * 2.0 ** -32
            u = torch.from_numpy(u.astype(np.float32))
            score = x - torch.log(-torch.log(u))
        score = torch.where(keep, score, torch.full_like(score, -math.inf))
        tok = int(torch.argmax(score))
        toks[b] = tok
        lps[b] = x[tok] - logz
        masks[b] = keep
    return toks, lps, masks


def pack_mask(mask):
    """bool [B, V] -> int32 bit words [B, ceil(V/32)] (bit i of word i//32)."""
    B, V = mask.shape
    W = (V + 31) // 32
    pad = torch.zeros(B, W * 32, dtype=torch.bool)
    pad[:, :V] = mask.cpu()
    bits = pad.view(B, W, 32).to(torch.int64) << torch.arange(32, dtype=torch.int64)
    words = bits.sum(-1)
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words)
    return words.to(torch.int32)


def unpack_mask(words, V):
    B, W = words.shape
    w = words.to(torch.int64) & 0xFFFFFFFF
    bits = (w[:, :, None] >> torch.arange(32, dtype=torch.int64)) & 1
    return bits.view(B, W * 32)[:, :V].bool()


def repetition_penalty(logits, prev, penalty):
    for b in range(logits.shape[0]):
        pen = float(penalty[b])
        if pen == 1.0:
            continue
        for tid in set(int(t) for t in prev[b].tolist() if 0 <= int(t) < logits.shape[1]):
            x = float(logits[b, tid])
            logits[b, tid] = x / pen if x > 0 else x * pen
    return logits


def mla_decode(q, cache, block_tables, row_seq, row_ctx, scale):
    """Absorbed-form latent attention. q [rows, H, 576] (512 latent | 64 rope), cache
    [blocks, 16, 576]; row r attends to the first row_ctx[r] latent rows of its
    sequence -> o_lat [rows, H, 512] = softmax(q . row * scale) @ row[:, :512]."""
    rows, H, _ = q.shape
    out = torch.zeros(rows, H, 512, dtype=q.dtype, device=q.device)
    for r in range(rows):
        n = int(row_ctx[r])
        if n == 0:
            continue
        bt = block_tables[int(row_seq[r])]
        idx = torch.arange(n, device=cache.device)
        rows_kv = cache[bt[(idx // BLOCK).long()].long(), idx % BLOCK].float()  # [n, 576]
        s = (q[r].float() @ rows_kv.t()) * scale
        out[r] = (torch.softmax(s, -1) @ rows_kv[:, :512]).to(q.dtype)
    return out
