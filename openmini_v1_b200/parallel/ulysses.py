"""Sequence parallelism by head / sequence all-to-all (the "Ulysses" scheme).

Rank r of W holds tokens [r C, (r+1) C) of a sequence with all H query heads and
all Hkv KV heads (H and Hkv divisible by W). One all-to-all per tensor turns this
into every token of the sequence for heads [r H/W, (r+1) H/W) (and the matching KV
heads). Each rank then runs ordinary causal attention over the whole sequence for
its head group: the FlashAttention kernel on the GPU, fp32 math on the CPU. A last
all-to-all returns the output to the sequence split. Per rank and layer this moves
4 x C x (H + 2 Hkv) / W x D values, which does not grow with W, against ring
attention's (W - 1) KV-chunk hops. Grouped-query attention is kept: query head h
reads KV head h // (H / Hkv), and both head groups are split contiguously.

The survey marks this strategy optional; the reference has no counterpart (its
sequence-parallel mode is an enum plus a warning,
openmini-server/src/model/inference/distributed_inference_engine.rs:356-358).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .ring_attention import attend


def _a2a(x: torch.Tensor, group) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty_like(x)  # after contiguous(): a dense output, not the view's strides
    dist.all_to_all_single(out, x, group=group)
    return out


def _seq_to_heads(x: torch.Tensor, W: int, group) -> torch.Tensor:
    """[C, Hx, D] (sequence chunk, all heads) -> [W C, Hx / W, D] (whole sequence, head group)."""
    C, Hx, D = x.shape
    send = x.view(C, W, Hx // W, D).transpose(0, 1)          # [dst rank, C, Hx / W, D]
    return _a2a(send, group).reshape(W * C, Hx // W, D)      # rows arrive in source-rank = sequence order


def _heads_to_seq(x: torch.Tensor, W: int, group) -> torch.Tensor:
    """[W C, Hx / W, D] -> [C, Hx, D]."""
    T, Hg, D = x.shape
    C = T // W
    back = _a2a(x.view(W, C, Hg, D), group)                  # [source head group, C, Hg, D]
    return back.transpose(0, 1).reshape(C, W * Hg, D)


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None,
                      group=None, causal: bool = True) -> torch.Tensor:
    """q [C, H, D], k / v [C, Hkv, D]: this rank's contiguous sequence chunk (equal C on
    every rank). Returns this chunk's attention output [C, H, D] in q's dtype."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    W = dist.get_world_size(group) if dist.is_initialized() else 1
    if W == 1:
        out, _ = attend(q, k, v, scale, causal=causal)
        return out.to(q.dtype)
    H, Hkv = q.shape[1], k.shape[1]
    if H % W or Hkv % W:
        raise ValueError(f"query heads ({H}) and KV heads ({Hkv}) must divide by the group size {W}")
    qh, kh, vh = (_seq_to_heads(t, W, group) for t in (q, k, v))
    out, _ = attend(qh, kh, vh, scale, causal=causal)
    return _heads_to_seq(out.to(q.dtype).contiguous(), W, group)
