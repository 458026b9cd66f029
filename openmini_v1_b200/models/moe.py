"""Mixture-of-experts FFN: router -> top-k -> softmax over the k logits ->
SwiGLU experts -> weighted combine.

Routing follows the reference's top_k_selection (top-k first, then softmax over
the selected logits; openmini-server/src/model/inference/model.rs:1325 and
813-960). Keep-Routing replay (openmini-server/src/rl/keep_routing.rs:113-180)
is supported by ``ForwardBatch.forced_routing[layer] = expert ids [T, k]``:
the forward then uses those experts (weights recomputed from the current
router so gradients still flow), and ``record_routing`` captures the ids the
router chose.
"""
from __future__ import annotations

import torch

from .. import ops


def route(router_logits: torch.Tensor, k: int, forced: torch.Tensor | None = None):
    """Returns (expert ids [T, k] int64, weights [T, k] fp32)."""
    lg = router_logits.float()
    if forced is not None:
        ids = forced.long()
        sel = lg.gather(1, ids)
    else:
        sel, ids = torch.topk(lg, k, dim=-1)
    w = torch.softmax(sel, dim=-1)
    return ids, w


def _stacked(L):
    """Experts' weights stacked [E, N, K] for the grouped GEMM (rebuilt when the lists change)."""
    src = (L["experts_gate_up"], L["experts_down"])
    if L.get("_stack_src") is not src:
        L["_gu_stack"] = torch.stack(list(src[0])).contiguous()
        L["_down_stack"] = torch.stack(list(src[1])).contiguous()
        L["_stack_src"] = src
    return L["_gu_stack"], L["_down_stack"]


def moe_forward_device(model, layer_idx, L, x, fb):
    """Graph-capturable MoE: device routing, expert-sorted rows, two grouped tcgen05 GEMMs, combine."""
    from .. import _native
    cfg = model.cfg.moe
    T, D = x.shape
    k, E = cfg.top_k, cfg.num_experts
    C = _native.C()
    dev = x.device
    logits = ops.linear(x, L["router"])
    forced = fb.forced_routing.get(layer_idx) if fb.forced_routing else None
    ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    w = torch.empty(T, k, dtype=torch.float32, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    C.moe_route(logits.contiguous(), k, forced.to(torch.int32).contiguous() if forced is not None else None,
                ids, w, counts)
    if fb.record_routing is not None:
        fb.record_routing[layer_idx] = ids.clone()
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    cursor = torch.empty(E, dtype=torch.int32, device=dev)
    row_of = torch.empty(T * k, dtype=torch.int32, device=dev)
    xp = torch.empty(T * k, D, dtype=x.dtype, device=dev)
    C.moe_permute(x.contiguous(), ids, counts, offsets, cursor, row_of, xp)
    gu_w, down_w = _stacked(L)
    status = ops.ctx(dev).status
    gu = torch.empty(T * k, gu_w.shape[1], dtype=x.dtype, device=dev)
    C.grouped_gemm(xp, gu_w, offsets, gu, status)
    act = ops.silu_mul(gu)
    yp = torch.empty(T * k, D, dtype=x.dtype, device=dev)
    C.grouped_gemm(act.contiguous(), down_w, offsets, yp, status)
    out = torch.empty(T, D, dtype=x.dtype, device=dev)
    C.moe_combine(yp, row_of, w, out, False)
    return out


def load_balance_loss(router_logits: torch.Tensor, ids: torch.Tensor, num_experts: int) -> torch.Tensor:
    """Switch-style auxiliary loss E * sum_e f_e * P_e: f_e the fraction of (token, choice)
    pairs routed to expert e, P_e the mean router probability of e (reference: MoE v2
    load-balance loss, openmini-server/src/model/inference/gguf.rs:1298)."""
    probs = torch.softmax(router_logits.float(), -1)[:, :num_experts]
    f = torch.bincount(ids.reshape(-1).clamp(max=num_experts), minlength=num_experts + 1)[:num_experts].float()
    f = f / max(1, ids.numel())
    return num_experts * (f * probs.mean(0)).sum()


def moe_forward(model, layer_idx, L, x, fb):
    """Routed experts (+ zero-computation experts) + shared experts."""
    y = _routed(model, layer_idx, L, x, fb)
    if "shared_gate_up" in L:
        y = y + ops.linear(ops.silu_mul(ops.linear(x, L["shared_gate_up"])), L["shared_down"])
    return y


def _routed(model, layer_idx, L, x, fb):
    cfg = model.cfg.moe
    T, D = x.shape
    ep = getattr(model, "_ep", None)
    if ep is not None and ep.size > 1:  # expert parallel: all-to-all dispatch / combine
        return ep.forward(model, layer_idx, L, x, fb)
    if (x.is_cuda and cfg.num_zero_experts == 0 and isinstance(L["experts_gate_up"][0], torch.Tensor)
            and x.dtype == torch.bfloat16
            and D % 64 == 0 and cfg.expert_ffn % 64 == 0 and cfg.num_experts <= 256 and cfg.top_k <= 8):
        return moe_forward_device(model, layer_idx, L, x, fb)
    logits = ops.linear(x, L["router"])
    forced = fb.forced_routing.get(layer_idx) if fb.forced_routing else None
    ids, w = route(logits, cfg.top_k, forced)
    if fb.record_routing is not None:
        fb.record_routing[layer_idx] = ids.to(torch.int32)
    out = torch.zeros(T, D, dtype=torch.float32, device=x.device)
    flat = ids.reshape(-1)
    tok = torch.arange(T, device=x.device).repeat_interleave(cfg.top_k)
    wt = w.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=cfg.num_experts + cfg.num_zero_experts).tolist()
    start = 0
    E = cfg.num_experts
    for e, n in enumerate(counts):
        if n == 0:
            continue
        sel = order[start:start + n]
        start += n
        t_idx = tok[sel]
        if e >= E:  # zero-computation expert: passes its tokens through, weighted
            out.index_add_(0, t_idx, x.index_select(0, t_idx).float() * wt[sel, None])
            continue
        xe = x.index_select(0, t_idx)
        gu = ops.linear(xe, L["experts_gate_up"][e])
        y = ops.linear(ops.silu_mul(gu), L["experts_down"][e])
        out.index_add_(0, t_idx, y.float() * wt[sel, None])
    return out.to(x.dtype)
