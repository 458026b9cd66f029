"""Differentiable wrappers of the native kernels for training.

``linear(x, w)`` computes x @ w^T with the tcgen05 GEMM on CUDA in forward
and backward (dX = dY @ W, dW = dY^T @ X, each expressed as the kernel's
x @ w^T form on transposed copies); on the CPU it is the fp32 torch statement.
"""
from __future__ import annotations

import torch

from .. import ops


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        return ops.linear(x, w)

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        gy = gy.contiguous().to(x.dtype)
        gx = gw = None
        if ctx.needs_input_grad[0]:
            padn = (-gy.shape[1]) % 8  # the output dim becomes the reduction dim (e.g. a 4-expert router)
            g2 = torch.nn.functional.pad(gy, (0, padn)) if padn else gy
            wt = torch.nn.functional.pad(w.t(), (0, padn)) if padn else w.t()
            gx = ops.linear(g2, wt.contiguous())                          # [M, K] = dY @ W
        if ctx.needs_input_grad[1]:
            pad = (-x.shape[0]) % 8  # the token dim becomes the reduction dim: keep rows 16-byte aligned
            xp = torch.nn.functional.pad(x, (0, 0, 0, pad)) if pad else x
            gp = torch.nn.functional.pad(gy, (0, 0, 0, pad)) if pad else gy
            gw = ops.linear(gp.t().contiguous(), xp.t().contiguous())     # [N, K] = dY^T @ X
        return gx, gw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        return x @ w.t()
    shp = x.shape
    y = _Linear.apply(x.reshape(-1, shp[-1]).contiguous(), w)
    return y.reshape(*shp[:-1], w.shape[0])


def rmsnorm(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


class _Attention(torch.autograd.Function):
    """Causal attention of q [B, T, H, D] over k, v [B, T, Hkv, D].

    Forward: the repo's attention per sequence (``parallel.ring_attention.attend``: the
    tcgen05 FlashAttention kernel on CUDA for head_dim 128, the fp32 statement on CPU),
    which also returns the natural-log sum of exponentials L of every row.
    Backward (flash-attention gradient from L, no stored probabilities):
        P = exp(scale q k^T - L),  dV = P^T dO,  dP = dO V^T,
        delta = rowsum(dO * O),    dS = P * (dP - delta),
        dQ = scale dS K,           dK = scale dS^T Q   (GQA: summed over each KV head's queries)."""

    @staticmethod
    def forward(ctx, q, k, v, scale):
        from ..parallel.ring_attention import attend
        B = q.shape[0]
        outs, lses = [], []
        for b in range(B):
            o, lse = attend(q[b].contiguous(), k[b].contiguous(), v[b].contiguous(), scale, causal=True)
            outs.append(o)
            lses.append(lse)
        out = torch.stack(outs)                    # fp32 [B, T, H, D]
        lse = torch.stack(lses)                    # [B, T, H]
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.scale = scale
        return out.to(q.dtype)

    @staticmethod
    def backward(ctx, go):
        q, k, v, out, lse = ctx.saved_tensors
        scale = ctx.scale
        B, T, H, D = q.shape
        Hkv = k.shape[2]
        G = H // Hkv
        qf, gof = q.float(), go.float()
        kf = k.float().repeat_interleave(G, dim=2)
        vf = v.float().repeat_interleave(G, dim=2)
        s = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * scale
        causal = torch.ones(T, T, dtype=torch.bool, device=q.device).triu(1)
        p = torch.exp(s - lse.permute(0, 2, 1)[..., None]).masked_fill(causal, 0.0)
        dv = torch.einsum("bhqk,bqhd->bkhd", p, gof)
        dp = torch.einsum("bqhd,bkhd->bhqk", gof, vf)
        delta = (gof * out).sum(-1).permute(0, 2, 1)[..., None]   # [B, H, T, 1]
        ds = p * (dp - delta)
        dq = torch.einsum("bhqk,bkhd->bqhd", ds, kf) * scale
        dk = torch.einsum("bhqk,bqhd->bkhd", ds, qf) * scale
        if G > 1:
            dk = dk.view(B, T, Hkv, G, D).sum(3)
            dv = dv.view(B, T, Hkv, G, D).sum(3)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """Differentiable causal attention, q [B, T, H, D], k / v [B, T, Hkv, D] -> [B, T, H, D]."""
    return _Attention.apply(q, k, v, scale)
