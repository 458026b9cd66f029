"""Expert parallelism for the MoE FFN: all-to-all dispatch -> local experts -> all-to-all combine.

With ``ep`` ranks in an expert-parallel group, rank r owns experts
[r E/ep, (r+1) E/ep). Every rank routes its own tokens with the replicated
router (top-k, then softmax over the k logits, exactly as the single-rank MoE),
then

  1. dispatch: each (token, choice) pair is sent to the rank owning its expert
     (one all_to_all_single of the token rows, one of the local expert ids;
     the per-destination counts are exchanged first),
  2. the owner runs its experts over the rows it received (grouped by expert),
  3. combine: the expert outputs go back with the reverse all-to-all and are
     summed into their tokens with the routing weights.

Keep-Routing replay works unchanged: forced expert ids enter at step 1.
On GPUs the all-to-alls run on NCCL over NVLink; on CPU on gloo (tests).

Reference counterpart: the MoE config (openmini-server/src/config/settings.rs:189-245)
and the local expert loop (openmini-server/src/model/inference/model.rs:813-960);
the reference has no expert parallelism.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from ..models.moe import route


def shard_experts(L: dict, ep: int, ep_rank: int) -> dict:
    """This rank's expert slice of a full MoE layer dict (router kept whole)."""
    E = len(L["experts_gate_up"])
    if E % ep:
        raise ValueError(f"{E} experts not divisible by ep={ep}")
    n = E // ep
    out = dict(L)
    out["experts_gate_up"] = L["experts_gate_up"][ep_rank * n:(ep_rank + 1) * n]
    out["experts_down"] = L["experts_down"][ep_rank * n:(ep_rank + 1) * n]
    for k in ("_gu_stack", "_down_stack", "_stack_src"):
        out.pop(k, None)
    return out


class ExpertParallel:
    """All-to-all expert parallelism over ``group`` (None = world)."""

    def __init__(self, group=None):
        self.group = group
        self.size = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def _a2a(self, send: torch.Tensor, in_splits: list, out_splits: list) -> torch.Tensor:
        out = send.new_empty((sum(out_splits),) + tuple(send.shape[1:]))
        dist.all_to_all_single(out, send.contiguous(), out_splits, in_splits, group=self.group)
        return out

    def forward(self, model, layer_idx: int, L: dict, x: torch.Tensor, fb) -> torch.Tensor:
        cfg = model.cfg.moe
        T, D = x.shape
        k, E, W = cfg.top_k, cfg.num_experts, self.size
        n_local = E // W
        if cfg.num_zero_experts:
            raise NotImplementedError("zero-computation experts are routed locally; use ep=1 for such layers")
        logits = ops.linear(x, L["router"])
        forced = fb.forced_routing.get(layer_idx) if fb is not None and fb.forced_routing else None
        ids, w = route(logits, k, forced)
        if fb is not None and fb.record_routing is not None:
            fb.record_routing[layer_idx] = ids.to(torch.int32)
        flat = ids.reshape(-1)
        tok = torch.arange(T, device=x.device).repeat_interleave(k)
        dest = flat // n_local
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=W)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        in_splits, out_splits = send_counts.tolist(), recv_counts.tolist()
        # 1. dispatch rows and their local expert ids
        rows = self._a2a(x.index_select(0, tok[order]), in_splits, out_splits)
        lid = self._a2a((flat[order] % n_local).to(torch.int64), in_splits, out_splits)
        # 2. local experts over the received rows
        y = torch.empty(rows.shape[0], D, dtype=x.dtype, device=x.device)
        if rows.shape[0]:
            eorder = torch.argsort(lid, stable=True)
            ecounts = torch.bincount(lid, minlength=n_local).tolist()
            s = 0
            for e, n in enumerate(ecounts):
                if n == 0:
                    continue
                sel = eorder[s:s + n]
                s += n
                gu = ops.linear(rows.index_select(0, sel), L["experts_gate_up"][e])
                y.index_copy_(0, sel, ops.linear(ops.silu_mul(gu), L["experts_down"][e]))
        # 3. combine: reverse all-to-all, weighted sum into the tokens
        back = self._a2a(y, out_splits, in_splits)
        out = torch.zeros(T, D, dtype=torch.float32, device=x.device)
        out.index_add_(0, tok[order], back.float() * w.reshape(-1)[order, None])
        return out.to(x.dtype)
