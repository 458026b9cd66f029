"""Sliding-window attention over the paged KV cache (Gemma-style local layers).

Row r (visible keys [0, ctx_r)) attends only to keys [max(0, ctx_r - W), ctx_r).
The window is a contiguous selection, so it runs on the sparse-gather attention
kernel of DSA (``dsa_attention``: per-row key index lists over the paged cache,
GQA, online softmax) with the index lists produced on the device; no second
attention kernel is needed. Rows whose context fits the window take the dense
paged kernels. KV of evicted positions stays in the cache (the block manager
still owns it), which keeps prefix sharing and preemption unchanged.

With ``sinks`` > 0 the first positions stay visible too (streaming attention with
attention sinks; reference: openmini-server/src/hardware/kv_cache/streaming.rs).

Reference counterpart: the sliding-window attention of the reference's Gemma-3
support (openmini-server/src/model/inference/sliding_window.rs).
"""
from __future__ import annotations

import torch

from .. import _native, ops
from .dsa import sparse_attention_ref


def window_indices(row_ctx: torch.Tensor, window: int, sinks: int = 0):
    """(sel int32 [rows, sinks + W], n int32 [rows]): the first ``sinks`` positions
    (streaming attention) followed by the window [ctx - W, ctx), without overlap."""
    ctx = row_ctx.to(torch.int32)
    start = torch.clamp(ctx - window, min=0)
    ar = torch.arange(window, dtype=torch.int32, device=ctx.device)[None, :]
    if sinks <= 0:
        return (start[:, None] + ar).contiguous(), (ctx - start).contiguous()
    s = torch.minimum(torch.full_like(start, sinks), start)       # sinks that precede the window
    sar = torch.arange(sinks, dtype=torch.int32, device=ctx.device)[None, :]
    sel = torch.cat([sar.expand(ctx.shape[0], sinks), start[:, None] + ar], 1)
    # compact: window entries move left over the unused sink slots
    idx = torch.arange(sinks + window, device=ctx.device)[None, :]
    src = torch.where(idx < s[:, None], idx, idx - s[:, None] + sinks)
    sel = torch.gather(sel, 1, src.clamp(max=sinks + window - 1).long())
    return sel.contiguous(), (s + ctx - start).contiguous()


def window_attention(model, qkv, kv_k, kv_v, fb, window: int, sinks: int = 0):
    if fb.max_ctx <= window + sinks:  # every row sees its whole context: dense kernels
        if fb.prefill_tiles is not None and model.hd == 128 and qkv.is_cuda:
            return ops.flash_prefill(qkv, kv_k, kv_v, fb.block_tables, fb.row_seq, fb.row_ctx, fb.prefill_tiles,
                                     model.hq, model.scale)
        return ops.paged_attention(qkv, kv_k, kv_v, fb.block_tables, fb.row_seq, fb.row_ctx, model.hq, model.scale,
                                   fb.max_ctx)
    sel, n = window_indices(fb.row_ctx, window, sinks)
    T = qkv.shape[0]
    if qkv.is_cuda:
        out = torch.empty(T, model.hq * model.hd, dtype=qkv.dtype, device=qkv.device)
        _native.C().dsa_attention(qkv, kv_k, kv_v, fb.block_tables, fb.row_seq, sel, n, out, model.hq, model.scale)
        return out
    return sparse_attention_ref(qkv, kv_k, kv_v, fb.block_tables, fb.row_seq, sel, n, model.hq, model.scale)
