"""Trainable policy for RL / supervised training.

Holds fp32 master parameters (``nn.Parameter``) of a decoder with the same
architecture and weight layout as :class:`DecoderLM`, computes in bf16 on the
GPU through the differentiable tcgen05 GEMM (``ops.autograd.linear``) and the
differentiable FlashAttention (``ops.autograd.attention``: tcgen05 kernel forward,
gradient recomputed from its log-sum-exp), and can
push its weights into an inference ``DecoderLM`` (rollout weight sync).

The forward takes whole sequences (no paged cache) and supports Keep-Routing
replay: ``forced_routing[layer] = expert ids [B*T, k]`` makes each MoE layer
use the rollout's experts while the routing weights still come from the
current router (so the router keeps receiving gradient).

Reference: MultimodalTransformer::forward_train / trainable_params
(openmini-server/src/model/inference/model.rs:4411-4553).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import autograd as ag
from ..ops import reference as ref
from .config import ModelConfig
from .moe import route


class Policy(nn.Module):
    def __init__(self, cfg: ModelConfig, device="cpu", seed: int = 0, std: float = 0.02,
                 compute_dtype=torch.bfloat16):
        super().__init__()
        self.cfg = cfg
        self.device = torch.device(device)
        self.cdt = compute_dtype if self.device.type == "cuda" else torch.float32
        g = torch.Generator().manual_seed(seed)
        D, hd = cfg.hidden_size, cfg.head_dim

        def P(*shape, ones=False):
            t = torch.ones(*shape) if ones else torch.randn(*shape, generator=g) * std
            return nn.Parameter(t.to(self.device))

        self.embed = P(cfg.vocab_size, D)
        self.norm = P(D, ones=True)
        self.lm_head = P(cfg.vocab_size, D)
        self.layers = nn.ModuleList()
        for i in range(cfg.num_layers):
            L = nn.Module()
            L.attn_norm, L.ffn_norm = P(D, ones=True), P(D, ones=True)
            L.qkv = P((cfg.num_heads + 2 * cfg.num_kv_heads) * hd, D)
            L.o = P(D, cfg.num_heads * hd)
            L.is_moe = cfg.moe.is_moe_layer(i)
            if L.is_moe:
                E, Fe = cfg.moe.num_experts, cfg.moe.expert_ffn
                L.router = P(E, D)
                L.experts_gate_up = nn.ParameterList([P(2 * Fe, D) for _ in range(E)])
                L.experts_down = nn.ParameterList([P(D, Fe) for _ in range(E)])
            else:
                L.gate_up = P(2 * cfg.intermediate_size, D)
                L.down = P(D, cfg.intermediate_size)
            self.layers.append(L)
        self.inv_freq = ref.inv_freq(hd, cfg.rope_theta).to(self.device)

    # ------------------------------------------------------------------ forward
    def _w(self, p):
        return p.to(self.cdt)

    def forward(self, ids: torch.Tensor, forced_routing: dict | None = None, record_routing: dict | None = None):
        """ids [B, T] -> logits [B, T, V] (fp32)."""
        cfg = self.cfg
        B, T = ids.shape
        H, Hkv, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        pos = torch.arange(T, device=ids.device)
        x = F.embedding(ids, self._w(self.embed))
        for i, L in enumerate(self.layers):
            a = ag.rmsnorm(x, self._w(L.attn_norm), cfg.rms_eps)
            qkv = ag.linear(a, self._w(L.qkv))
            q = qkv[..., :H * hd].view(B, T, H, hd)
            k = qkv[..., H * hd:(H + Hkv) * hd].view(B, T, Hkv, hd)
            v = qkv[..., (H + Hkv) * hd:].view(B, T, Hkv, hd)
            q = _rope(q, pos, self.inv_freq, cfg.rope_mode)
            k = _rope(k, pos, self.inv_freq, cfg.rope_mode)
            o = ag.attention(q, k, v, 1.0 / math.sqrt(hd)).reshape(B, T, H * hd)
            x = x + ag.linear(o, self._w(L.o))
            h = ag.rmsnorm(x, self._w(L.ffn_norm), cfg.rms_eps)
            if L.is_moe:
                x = x + self._moe(i, L, h.reshape(B * T, -1), forced_routing, record_routing).view(B, T, -1)
            else:
                gu = ag.linear(h, self._w(L.gate_up))
                Fd = gu.shape[-1] // 2
                x = x + ag.linear(F.silu(gu[..., :Fd]) * gu[..., Fd:], self._w(L.down))
        x = ag.rmsnorm(x, self._w(self.norm), cfg.rms_eps)
        return ag.linear(x, self._w(self.lm_head)).float()

    def _moe(self, i, L, h, forced, record):
        k = self.cfg.moe.top_k
        logits = ag.linear(h, self._w(L.router))
        f = forced.get(i) if forced else None
        ids, w = route(logits, k, f)
        if record is not None:
            record[i] = ids.to(torch.int32)
        out = torch.zeros_like(h, dtype=torch.float32)
        flat = ids.reshape(-1)
        tok = torch.arange(h.shape[0], device=h.device).repeat_interleave(k)
        wt = w.reshape(-1)
        for e in range(self.cfg.moe.num_experts):
            sel = (flat == e).nonzero().flatten()
            if sel.numel() == 0:
                continue
            t_idx = tok[sel]
            gu = ag.linear(h.index_select(0, t_idx), self._w(L.experts_gate_up[e]))
            Fe = gu.shape[-1] // 2
            y = ag.linear(F.silu(gu[:, :Fe]) * gu[:, Fe:], self._w(L.experts_down[e]))
            out = out.index_add(0, t_idx, y.float() * wt[sel, None])
        return out.to(h.dtype)

    # ------------------------------------------------------------------ weight sync
    @torch.no_grad()
    def export_to(self, model):
        """Copy the current weights into an inference DecoderLM (same config, tp = 1)."""
        dt = model.dtype
        model.embed = self.embed.detach().to(dt).to(model.device)
        model.norm = self.norm.detach().to(dt).to(model.device)
        model.lm_head = self.lm_head.detach().to(dt).to(model.device)
        for L, M in zip(self.layers, model.layers):
            for name in ("attn_norm", "ffn_norm", "qkv", "o"):
                M[name] = getattr(L, name).detach().to(dt).to(model.device).contiguous()
            if L.is_moe:
                M["router"] = L.router.detach().to(dt).to(model.device).contiguous()
                M["experts_gate_up"] = [p.detach().to(dt).to(model.device).contiguous() for p in L.experts_gate_up]
                M["experts_down"] = [p.detach().to(dt).to(model.device).contiguous() for p in L.experts_down]
            else:
                M["gate_up"] = L.gate_up.detach().to(dt).to(model.device).contiguous()
                M["down"] = L.down.detach().to(dt).to(model.device).contiguous()


def _rope(x, pos, inv_f, mode):
    ang = pos.float()[:, None] * inv_f[None, :]
    c, s = torch.cos(ang)[None, :, None, :], torch.sin(ang)[None, :, None, :]
    xf = x.float()
    if mode == 0:
        x0, x1 = xf[..., 0::2], xf[..., 1::2]
        out = torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1).flatten(-2)
    else:
        h = x.shape[-1] // 2
        x0, x1 = xf[..., :h], xf[..., h:]
        out = torch.cat([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1)
    return out.to(x.dtype)


def token_logprobs(logits: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0, keep_mask=None):
    """log p(target) under softmax(logits / T), optionally restricted to a kept set (bool [.., V])."""
    lg = logits / max(temperature, 1e-6)
    if keep_mask is not None:
        lg = lg.masked_fill(~keep_mask, float("-inf"))
    return torch.log_softmax(lg, -1).gather(-1, targets.unsqueeze(-1)).squeeze(-1)
