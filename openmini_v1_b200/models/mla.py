"""Multi-head latent attention (MLA) layer of the decoder, absorbed form.

Per token the cache keeps one 576-wide row: the RMS-normed KV latent c (512) and
the rotated shared key part k_r (64), 1152 bytes in bf16 against 2 x heads x
head_dim x 2 bytes for ordinary KV (8 KB at 16 heads of 128). Per layer:

    q      = W_q x                       -> per head [q_nope (dn) | q_r (dr)]
    [c|k]  = W_dkv x;  c = RMSNorm(c);  k_r = RoPE(k)        (written to the cache)
    q_lat  = W_uk[h]^T q_nope[h]         -> 512    (up-projection absorbed into q)
    o_lat  = attention of [q_lat | RoPE(q_r)] over the cached rows (values = c)
    o[h]   = W_uv[h] o_lat[h]            -> dv, then the output projection

The attention runs on the paged latent cache in ``csrc/attn/mla.cu``
(``ops.mla_decode``); the projections are GEMMs. Under tensor parallelism the
heads (W_q rows, W_uk, W_uv, W_o columns) are split and W_dkv is replicated.

Reference counterpart: openmini-server/src/hardware/kv_cache/mla/{config,
projection,latent_cache,attention}.rs and model/inference/model.rs:962-1027
(MLAWeights), 2381-2712 (MLA forward). The reference caches latent_dim/2-wide
halves per KV head; this follows the published MLA layout (one shared latent row
with a decoupled RoPE key).
"""
from __future__ import annotations

import math

import torch

from .. import ops
from ..ops import reference as ref

LAT, ROPE = 512, 64


def init_mla(model, L: dict, gen, shared, std: float):
    cfg, m = model.cfg, model.cfg.mla
    D, H = cfg.hidden_size, model.hq
    if m.q_lora_rank:
        L["mla_q_a"] = model._randn(gen, m.q_lora_rank, D, std=std)
        L["mla_q_a_norm"] = torch.ones(m.q_lora_rank, dtype=model.dtype, device=model.device)
        L["mla_q_b"] = model._randn(gen, H * (m.qk_nope_dim + m.qk_rope_dim), m.q_lora_rank, std=std)
    else:
        L["mla_q"] = model._randn(gen, H * (m.qk_nope_dim + m.qk_rope_dim), D, std=std)
    L["mla_dkv"] = model._randn(shared, LAT + ROPE, D, std=std)
    L["mla_kv_norm"] = torch.ones(LAT, dtype=model.dtype, device=model.device)
    L["mla_uk"] = model._randn(gen, H, m.qk_nope_dim, LAT, std=std * 4)
    L["mla_uv"] = model._randn(gen, H, m.v_head_dim, LAT, std=std * 4)
    L["o"] = model._randn(gen, D, H * m.v_head_dim, std=std)


def mla_query(model, L: dict, a: torch.Tensor) -> torch.Tensor:
    """[T, D] -> [T, H (dn + dr)]: the full query projection, or the low-rank one
    (down-projection, RMSNorm, up-projection) when the checkpoint has it."""
    if "mla_q_a" in L:
        qa = ops.rmsnorm(ops.linear(a, L["mla_q_a"]), L["mla_q_a_norm"], model.cfg.rms_eps)
        return ops.linear(qa, L["mla_q_b"])
    return ops.linear(a, L["mla_q"])


def mla_scale(cfg) -> float:
    return 1.0 / math.sqrt(cfg.mla.qk_nope_dim + cfg.mla.qk_rope_dim)


def write_latent(cache: torch.Tensor, slots: torch.Tensor, rows: torch.Tensor):
    m = slots >= 0
    cache.view(-1, LAT + ROPE).index_copy_(0, slots[m].long(), rows[m].to(cache.dtype))


def mla_attention(model, i: int, L: dict, a: torch.Tensor, fb, kv) -> torch.Tensor:
    """a: normed hidden rows [T, D] -> attention output [T, H * dv] (before W_o)."""
    cfg, m = model.cfg, model.cfg.mla
    T, H, dn, dr = a.shape[0], model.hq, m.qk_nope_dim, m.qk_rope_dim
    q = mla_query(model, L, a).view(T, H, dn + dr)
    ck = ops.linear(a, L["mla_dkv"])
    c = ops.rmsnorm(ck[:, :LAT].contiguous(), L["mla_kv_norm"], cfg.rms_eps)
    k_r = ref.rope(ck[:, LAT:].reshape(T, 1, ROPE), fb.positions, model.mla_inv_freq, cfg.rope_mode).view(T, ROPE)
    write_latent(kv.k[i], fb.slots, torch.cat([c, k_r], dim=-1))
    q_r = ref.rope(q[..., dn:], fb.positions, model.mla_inv_freq, cfg.rope_mode)
    q_lat = torch.bmm(q[..., :dn].transpose(0, 1), L["mla_uk"]).transpose(0, 1)  # [T, H, 512]
    qa = torch.cat([q_lat, q_r.to(q_lat.dtype)], dim=-1).contiguous()
    o_lat = ops.mla_decode(qa, kv.k[i], fb.block_tables, fb.row_seq, fb.row_ctx, fb.max_ctx, mla_scale(cfg))
    o = torch.bmm(o_lat.transpose(0, 1), L["mla_uv"].transpose(1, 2))  # [H, T, dv]
    return o.transpose(0, 1).reshape(T, H * m.v_head_dim)


def mla_reference_layer(model, L: dict, a: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Unabsorbed fp32 statement of one causal MLA attention over a single sequence
    (keys k = [W_uk c | k_r] and values v = W_uv c per head), for tests."""
    cfg, m = model.cfg, model.cfg.mla
    T, H, dn = a.shape[0], model.hq, m.qk_nope_dim
    f = lambda t: t.float()
    if "mla_q_a" in L:
        qa = ref.rmsnorm(f(a) @ f(L["mla_q_a"]).t(), f(L["mla_q_a_norm"]), cfg.rms_eps).float()
        q = (qa @ f(L["mla_q_b"]).t()).view(T, H, -1)
    else:
        q = (f(a) @ f(L["mla_q"]).t()).view(T, H, -1)
    ck = f(a) @ f(L["mla_dkv"]).t()
    c = ref.rmsnorm(ck[:, :LAT], f(L["mla_kv_norm"]), cfg.rms_eps).float()
    k_r = ref.rope(ck[:, LAT:].reshape(T, 1, ROPE), positions, model.mla_inv_freq, cfg.rope_mode).float()
    q_r = ref.rope(q[..., dn:], positions, model.mla_inv_freq, cfg.rope_mode).float()
    k_nope = torch.einsum("tr,hdr->thd", c, f(L["mla_uk"]))
    v = torch.einsum("tr,hdr->thd", c, f(L["mla_uv"]))
    s = (torch.einsum("qhd,khd->hqk", q[..., :dn], k_nope) + torch.einsum("qhd,kd->hqk", q_r, k_r[:, 0])) \
        * mla_scale(cfg)
    s = s + torch.full((T, T), float("-inf"), device=a.device).triu(1)
    o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v)
    return o.reshape(T, -1)
