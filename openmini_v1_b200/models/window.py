"""Sliding-window attention over the paged KV cache (Gemma-style local layers).

Row r (visible keys [0, ctx_r)) attends only to keys [max(0, ctx_r - W), ctx_r).
The window is a contiguous selection, so it runs on the sparse-gather attention
kernel of DSA (``dsa_attention``: per-row key index lists over the paged cache,
GQA, online softmax) with the index lists produced on the device; no second
attention kernel is needed. Rows whose context fits the window take the dense
paged kernels. KV of evicted positions stays in the cache (the block manager
still owns it), which keeps prefix sharing and preemption unchanged.

Reference counterpart: the sliding-window attention of the reference's Gemma-3
support (openmini-server/src/model/inference/sliding_window.rs).
"""
from __future__ import annotations

import torch

from .. import _native, ops
from .dsa import sparse_attention_ref


def window_indices(row_ctx: torch.Tensor, window: int):
    """(sel int32 [rows, W], n int32 [rows]): key positions [ctx - W, ctx) clipped at 0."""
    ctx = row_ctx.to(torch.int32)
    start = torch.clamp(ctx - window, min=0)
    sel = start[:, None] + torch.arange(window, dtype=torch.int32, device=ctx.device)[None, :]
    n = ctx - start
    return sel.contiguous(), n.contiguous()


def window_attention(model, qkv, kv_k, kv_v, fb, window: int):
    if fb.max_ctx <= window:  # every row sees its whole context: dense kernels
        if fb.prefill_tiles is not None and model.hd == 128 and qkv.is_cuda:
            return ops.flash_prefill(qkv, kv_k, kv_v, fb.block_tables, fb.row_seq, fb.row_ctx, fb.prefill_tiles,
                                     model.hq, model.scale)
        return ops.paged_attention(qkv, kv_k, kv_v, fb.block_tables, fb.row_seq, fb.row_ctx, model.hq, model.scale,
                                   fb.max_ctx)
    sel, n = window_indices(fb.row_ctx, window)
    T = qkv.shape[0]
    if qkv.is_cuda:
        out = torch.empty(T, model.hq * model.hd, dtype=qkv.dtype, device=qkv.device)
        _native.C().dsa_attention(qkv, kv_k, kv_v, fb.block_tables, fb.row_seq, sel, n, out, model.hq, model.scale)
        return out
    return sparse_attention_ref(qkv, kv_k, kv_v, fb.block_tables, fb.row_seq, sel, n, model.hq, model.scale)
