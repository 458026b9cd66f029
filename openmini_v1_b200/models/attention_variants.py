"""Experimental attention variants for long contexts, written for one sequence
(causal unless stated) over q [T, H, D] and k, v [T, Hkv, D] (GQA: H a multiple of
Hkv), computed in fp32. They are the building blocks the decoder's configuration
can route long prompts through; each is tested against full attention on the
configuration where the two must agree.

* ``nsa_attention``: Native Sparse Attention. Three branches: attention over
  block-compressed keys (mean of each block of ``block`` keys), over the top-``n_sel``
  key blocks chosen from the compressed scores (summed over the query heads of a KV
  head, the first and the current block always kept), and over a sliding window.
  Per-head gates (sigmoid of a projection of q, or equal thirds) mix them.
* ``kascade_indices`` / ``KascadeCache`` / ``sparse_attention``: Kascade. Exact top-k
  key indices are computed only at anchor layers (every ``anchor_interval``) and
  reused by the layers between; attention then runs over the selected keys.
* ``tpa_project`` / ``TPACache``: Tensor Product Attention. Q, K, V are rank-R sums
  of outer products head-factor (x) feature-factor; the cache keeps the factors
  (R (H + D) per token instead of H D).
* ``sinkhorn_attention``: multi-head Sinkhorn (mHC). Alternating row / column
  normalisation of exp(scores) towards a doubly stochastic matrix (bidirectional).
* ``attn_res``: Attention Residuals. The residual of layer l is x_0 plus a softmax-
  weighted sum over earlier block summaries, weights from w_l . RMSNorm(summary).
* ``ahn_attention``: AHN. Tokens inside a sliding window get exact attention; tokens
  that left it are compressed into a linear-attention state (feature map elu + 1);
  a per-head gate mixes the two.
* ``linear_attention``: causal linear attention in chunked form (exact against the
  token-by-token recurrence), the long-context path of a ring / flash / linear hybrid.
* ``fp8_kv_quantize`` / ``fp8_kv_dequantize``: KV blocks as e4m3 with one fp32 scale
  per (block, head).

Reference counterparts: openmini-server/src/model/inference/{nsa,kascade,tpa,mhc,
attn_res,ahn}.rs and ring_flash_linear.rs:805-1245 (linear-attention path, FP8 KV).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _expand(k: torch.Tensor, H: int) -> torch.Tensor:
    return k.float().repeat_interleave(H // k.shape[1], dim=1)


def full_attention(q, k, v, scale=None, causal=True):
    T, H, D = q.shape
    scale = scale or 1 / math.sqrt(D)
    s = torch.einsum("thd,shd->hts", q.float(), _expand(k, H)) * scale
    if causal:
        s = s + torch.full((T, k.shape[0]), float("-inf"), device=q.device).triu(1 + k.shape[0] - T)
    return torch.einsum("hts,shd->thd", torch.softmax(s, -1), _expand(v, H))


def _masked_attention(q, k, v, mask, scale):
    """mask [H or 1, T, S] bool (True = visible)."""
    H = q.shape[1]
    s = torch.einsum("thd,shd->hts", q.float(), _expand(k, H)) * scale
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, -1)
    p = torch.nan_to_num(p, nan=0.0)  # rows with nothing visible
    return torch.einsum("hts,shd->thd", p, _expand(v, H))


# ----------------------------------------------------------------------------- NSA

def nsa_attention(q, k, v, block: int = 32, n_sel: int = 16, window: int = 512, gate_w=None, scale=None):
    T, H, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    scale = scale or 1 / math.sqrt(D)
    dev = q.device
    t = torch.arange(T, device=dev)
    nb = (T + block - 1) // block
    # compressed branch: block j visible to query t once the block is complete (end <= t + 1)
    pad = nb * block - T
    kp = F.pad(k.float(), (0, 0, 0, 0, 0, pad)).view(nb, block, Hkv, D)
    vp = F.pad(v.float(), (0, 0, 0, 0, 0, pad)).view(nb, block, Hkv, D)
    cnt = torch.clamp(T - torch.arange(nb, device=dev) * block, max=block).float()
    kc = kp.sum(1) / cnt[:, None, None]
    vc = vp.sum(1) / cnt[:, None, None]
    blk_end = (torch.arange(nb, device=dev) + 1) * block
    cmask = (blk_end[None, :] <= t[:, None] + 1)[None]
    o_cmp = _masked_attention(q, kc, vc, cmask, scale)
    # selection: block importance from compressed scores, summed over each KV head's group
    sc = torch.einsum("thd,jhd->htj", q.float(), _expand(kc, H)) * scale
    sc = sc.masked_fill(~cmask, float("-inf"))
    imp = torch.softmax(sc, -1).nan_to_num(0.0).view(Hkv, G, T, nb).sum(1)  # [Hkv, T, nb]
    cur = (t // block)
    imp[:, t, cur] = float("inf")      # the current (partial) block
    imp[:, :, 0] = float("inf")        # the first block
    future = torch.arange(nb, device=dev)[None, :] > cur[:, None]
    imp = imp.masked_fill(future[None], float("-inf"))
    n = min(n_sel, nb)
    top = imp.topk(n, dim=-1).indices                                  # [Hkv, T, n]
    sel_blocks = torch.zeros(Hkv, T, nb, dtype=torch.bool, device=dev)
    sel_blocks.scatter_(-1, top, True)
    sel_blocks &= ~future[None]
    tok_block = torch.arange(T, device=dev) // block
    smask = sel_blocks[:, :, tok_block] & (t[None, None, :] <= t[None, :, None])   # [Hkv, T, S]
    o_sel = _masked_attention(q, k, v, smask.repeat_interleave(G, dim=0), scale)
    # sliding window branch
    wmask = ((t[None, :] <= t[:, None]) & (t[None, :] > t[:, None] - window))[None]
    o_win = _masked_attention(q, k, v, wmask, scale)
    if gate_w is None:
        g = torch.full((T, H, 3), 1.0 / 3, device=dev)
    else:  # gate_w [H * 3, D]: per head and branch from that head's query
        g = torch.sigmoid(torch.einsum("thd,hbd->thb", q.float(), gate_w.float().view(H, 3, D)))
    return g[..., 0:1] * o_cmp + g[..., 1:2] * o_sel + g[..., 2:3] * o_win


# ----------------------------------------------------------------------------- Kascade

def kascade_indices(q, k, top_k: int):
    """Exact top-k key indices per query row (scores summed over heads, causal): [T, k]
    with -1 where a row has fewer visible keys."""
    T, H, _ = q.shape
    s = torch.einsum("thd,shd->ts", q.float(), _expand(k, H))
    s = s + torch.full((T, k.shape[0]), float("-inf"), device=q.device).triu(1)
    kk = min(top_k, k.shape[0])
    val, idx = s.topk(kk, dim=-1)
    return torch.where(torch.isfinite(val), idx, torch.full_like(idx, -1))


def sparse_attention(q, k, v, idx, scale=None):
    """Attention of row t over keys idx[t] (-1 = none)."""
    T, H, D = q.shape
    scale = scale or 1 / math.sqrt(D)
    ok = idx >= 0
    ii = idx.clamp(min=0)
    K = _expand(k, H)[ii]   # [T, n, H, D]
    V = _expand(v, H)[ii]
    s = torch.einsum("thd,tnhd->thn", q.float(), K) * scale
    s = s.masked_fill(~ok[:, None, :], float("-inf"))
    return torch.einsum("thn,tnhd->thd", torch.softmax(s, -1).nan_to_num(0.0), V)


class KascadeCache:
    """Anchor layers (0, interval, 2 interval, ...) compute indices; the layers in between
    reuse the latest anchor's. ``strategy``: "direct" reuses as is; "union" merges the
    two nearest anchors' selections (kept to the first top_k distinct keys)."""

    def __init__(self, num_layers: int, anchor_interval: int = 4, top_k: int = 2048, strategy: str = "direct"):
        self.L, self.every, self.top_k, self.strategy = num_layers, anchor_interval, top_k, strategy
        self.idx: dict = {}
        self.computed = 0

    def is_anchor(self, layer: int) -> bool:
        return layer % self.every == 0

    def anchors(self) -> list:
        return [i for i in range(self.L) if self.is_anchor(i)]

    def indices(self, layer: int, q, k):
        if self.is_anchor(layer):
            self.idx[layer] = kascade_indices(q, k, self.top_k)
            self.computed += 1
            return self.idx[layer]
        a = layer - layer % self.every
        sel = self.idx[a]
        if self.strategy == "union" and a - self.every in self.idx:
            both = torch.cat([sel, self.idx[a - self.every]], dim=-1)
            out = torch.full_like(sel, -1)
            for t in range(sel.shape[0]):
                u = [x for x in dict.fromkeys(both[t].tolist()) if x >= 0][: sel.shape[1]]
                out[t, :len(u)] = torch.tensor(u, dtype=sel.dtype)
            return out
        return sel


# ----------------------------------------------------------------------------- TPA

def tpa_project(x, wa, wb, H: int, D: int, R: int):
    """x [T, Dm]; wa [R H, Dm] head factors, wb [R D, Dm] feature factors ->
    [T, H, D] = (1/R) sum_r a_r (x) b_r, and the factors (a [T, R, H], b [T, R, D])."""
    T = x.shape[0]
    a = (x.float() @ wa.float().t()).view(T, R, H)
    b = (x.float() @ wb.float().t()).view(T, R, D)
    return torch.einsum("trh,trd->thd", a, b) / R, (a, b)


class TPACache:
    """Keeps the K / V factors of every position: decode reconstructs the keys from them."""

    def __init__(self):
        self.ka, self.kb, self.va, self.vb = [], [], [], []

    def append(self, kf, vf):
        self.ka.append(kf[0])
        self.kb.append(kf[1])
        self.va.append(vf[0])
        self.vb.append(vf[1])

    def kv(self):
        ka, kb = torch.cat(self.ka), torch.cat(self.kb)
        va, vb = torch.cat(self.va), torch.cat(self.vb)
        k = torch.einsum("trh,trd->thd", ka, kb) / ka.shape[1]
        v = torch.einsum("trh,trd->thd", va, vb) / va.shape[1]
        return k, v

    def floats_per_token(self) -> int:
        return sum(t.shape[1] * t.shape[2] for t in (self.ka[0], self.kb[0], self.va[0], self.vb[0]))


# ----------------------------------------------------------------------------- Sinkhorn (mHC)

def sinkhorn_attention(q, k, v, iters: int = 8, scale=None):
    T, H, D = q.shape
    scale = scale or 1 / math.sqrt(D)
    s = torch.einsum("thd,shd->hts", q.float(), _expand(k, H)) * scale
    logp = s - s.amax(dim=(-1, -2), keepdim=True)
    for _ in range(iters):  # in log space: rows then columns
        logp = logp - torch.logsumexp(logp, dim=-1, keepdim=True)
        logp = logp - torch.logsumexp(logp, dim=-2, keepdim=True)
    p = torch.softmax(logp, dim=-1)  # final row normalisation: outputs are convex combinations
    return torch.einsum("hts,shd->thd", p, _expand(v, H)), p


# ----------------------------------------------------------------------------- AttnRes

def attn_res(x0, summaries: list, w, eps: float = 1e-6):
    """h = x0 + sum_k softmax_k(w . RMSNorm(summary_k)) summary_k; summaries [T, D] each."""
    S = torch.stack([s.float() for s in summaries])                      # [K, T, D]
    n = S * torch.rsqrt(S.pow(2).mean(-1, keepdim=True) + eps)
    alpha = torch.softmax(torch.einsum("ktd,d->kt", n, w.float()), dim=0)  # over k
    return x0.float() + torch.einsum("kt,ktd->td", alpha, S), alpha


# ----------------------------------------------------------------------------- linear attention / AHN

def _phi(x):
    return F.elu(x) + 1.0


def linear_attention(q, k, v, chunk: int = 64):
    """Causal linear attention o_t = phi(q_t) S_t / phi(q_t) z_t, S_t = sum_{s<=t} phi(k_s)^T v_s,
    in chunks: inter-chunk state plus intra-chunk masked products."""
    T, H, D = q.shape
    qf, kf, vf = _phi(q.float()), _phi(_expand(k, H)), _expand(v, H)
    S = torch.zeros(H, D, vf.shape[-1], device=q.device)
    z = torch.zeros(H, D, device=q.device)
    out = torch.empty(T, H, vf.shape[-1], device=q.device)
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        qc, kc, vc = qf[c0:c1], kf[c0:c1], vf[c0:c1]
        n = c1 - c0
        m = torch.ones(n, n, device=q.device).tril()
        att = torch.einsum("thd,shd->hts", qc, kc) * m
        num = torch.einsum("thd,hde->the", qc, S) + torch.einsum("hts,she->the", att, vc)
        den = torch.einsum("thd,hd->th", qc, z) + att.sum(-1).transpose(0, 1)
        out[c0:c1] = num / den[..., None]
        S = S + torch.einsum("shd,she->hde", kc, vc)
        z = z + kc.sum(0)
    return out


def linear_attention_recurrent(q, k, v):
    T, H, D = q.shape
    qf, kf, vf = _phi(q.float()), _phi(_expand(k, H)), _expand(v, H)
    S = torch.zeros(H, D, vf.shape[-1])
    z = torch.zeros(H, D)
    out = []
    for t in range(T):
        S = S + torch.einsum("hd,he->hde", kf[t], vf[t])
        z = z + kf[t]
        out.append(torch.einsum("hd,hde->he", qf[t], S) / torch.einsum("hd,hd->h", qf[t], z)[:, None])
    return torch.stack(out)


def ahn_attention(q, k, v, window: int = 512, gate=None, scale=None):
    """Exact attention inside the window, linear-attention state for tokens older than it."""
    T, H, D = q.shape
    scale = scale or 1 / math.sqrt(D)
    t = torch.arange(T, device=q.device)
    wmask = ((t[None, :] <= t[:, None]) & (t[None, :] > t[:, None] - window))[None]
    local = _masked_attention(q, k, v, wmask, scale)
    qf, kf, vf = _phi(q.float()), _phi(_expand(k, H)), _expand(v, H)
    old = (t[None, :] <= t[:, None] - window).float()                     # [T, S] keys that left the window
    num = torch.einsum("thd,ts,shd,she->the", qf, old, kf, vf)
    den = torch.einsum("thd,ts,shd->th", qf, old, kf)
    has_old = den > 0
    rnn = torch.where(has_old[..., None], num / den.clamp(min=1e-30)[..., None], torch.zeros_like(num))
    g = torch.full((T, H, 1), 0.5, device=q.device) if gate is None else torch.sigmoid(gate.float())[None, :, None]
    g = torch.where(has_old[..., None], g, torch.ones_like(g))
    return g * local + (1 - g) * rnn


# ----------------------------------------------------------------------------- FP8 KV

def fp8_kv_quantize(cache: torch.Tensor):
    """[blocks, Hkv, 16, D] -> (e4m3 codes, fp32 scale [blocks, Hkv]) with amax / 448 per block and head."""
    amax = cache.float().abs().amax(dim=(2, 3)).clamp(min=1e-12)
    s = amax / 448.0
    codes = (cache.float() / s[:, :, None, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    return codes, s


def fp8_kv_dequantize(codes, s, dtype=torch.bfloat16):
    return (codes.float() * s[:, :, None, None]).to(dtype)
