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

Fixed-capacity mode (``capacity_factor`` set): every rank sends exactly C rows to
every rank (C = ceil(T k / W * capacity_factor)), so the all-to-alls have equal
splits and nothing waits for the host (C comes from ``max_tokens``, an agreed bound
on every rank's token count): each (token, choice) pair's slot is its
destination times C plus its position among the pairs for that destination
(a device cumsum); pairs past C are dropped (they contribute nothing to their
token, counted in ``dropped``). The owner sorts its received rows by local expert
on the device and runs the two grouped tcgen05 GEMMs of ``csrc/moe/moe.cu`` with
device offsets; the path is free of host synchronisation, so it can be captured
in a CUDA graph.

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

    def __init__(self, group=None, capacity_factor: float | None = None, max_tokens: int | None = None):
        self.group = group
        self.size = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.capacity_factor = capacity_factor
        self.max_tokens = max_tokens  # agreed bound on any rank's tokens (the capacity must match on all ranks)
        self.dropped = None  # device count of pairs dropped by the last fixed-capacity dispatch

    def _a2a(self, send: torch.Tensor, in_splits: list, out_splits: list) -> torch.Tensor:
        out = send.new_empty((sum(out_splits),) + tuple(send.shape[1:]))
        dist.all_to_all_single(out, send.contiguous(), out_splits, in_splits, group=self.group)
        return out

    def forward(self, model, layer_idx: int, L: dict, x: torch.Tensor, fb) -> torch.Tensor:
        if self.capacity_factor is not None:
            return self.forward_fixed(model, layer_idx, L, x, fb)
        return self.forward_exact(model, layer_idx, L, x, fb)

    def forward_fixed(self, model, layer_idx: int, L: dict, x: torch.Tensor, fb) -> torch.Tensor:
        import math
        cfg = model.cfg.moe
        T, D = x.shape
        k, E, W = cfg.top_k, cfg.num_experts, self.size
        n_local = E // W
        dev = x.device
        if cfg.num_zero_experts:
            raise NotImplementedError("zero-computation experts are routed locally; use ep=1 for such layers")
        Tb = self.max_tokens if self.max_tokens is not None else T
        if T > Tb:
            raise ValueError(f"{T} tokens exceed the expert-parallel max_tokens {Tb}")
        Cap = max(1, math.ceil(Tb * k / W * self.capacity_factor))
        logits = ops.linear(x, L["router"])
        forced = fb.forced_routing.get(layer_idx) if fb is not None and fb.forced_routing else None
        ids, w = route(logits, k, forced)
        if fb is not None and fb.record_routing is not None:
            fb.record_routing[layer_idx] = ids.to(torch.int32)
        flat = ids.reshape(-1)
        tok = torch.arange(T, device=dev).repeat_interleave(k)
        dest = flat // n_local
        onehot = torch.nn.functional.one_hot(dest, W)
        pos = (onehot.cumsum(0) - 1).gather(1, dest[:, None]).squeeze(1)
        keep = pos < Cap
        self.dropped = (~keep).sum()
        scratch = W * Cap  # dropped pairs land in one scratch row that is never sent
        slot = torch.where(keep, dest * Cap + pos, torch.full_like(pos, scratch))
        send = torch.zeros(scratch + 1, D, dtype=x.dtype, device=dev)
        send.index_copy_(0, slot, x.index_select(0, tok))
        sid = torch.full((scratch + 1,), -1, dtype=torch.int64, device=dev)
        sid.index_copy_(0, slot, flat % n_local)
        recv = torch.empty(scratch, D, dtype=x.dtype, device=dev)
        dist.all_to_all_single(recv, send[:scratch].contiguous(), group=self.group)
        rid = torch.empty(scratch, dtype=torch.int64, device=dev)
        dist.all_to_all_single(rid, sid[:scratch].contiguous(), group=self.group)
        y = self._local_experts(L, recv, rid, n_local)
        back = torch.empty(scratch + 1, D, dtype=x.dtype, device=dev)
        back[scratch].zero_()
        dist.all_to_all_single(back[:scratch], y, group=self.group)
        wk = w.reshape(-1) * keep.float()
        out = torch.zeros(T, D, dtype=torch.float32, device=dev)
        out.index_add_(0, tok, back.index_select(0, slot).float() * wk[:, None])
        return out.to(x.dtype)

    def _local_experts(self, L, rows, lid, n_local):
        """Rows [R, D] with local expert ids (-1 = empty slot) -> expert outputs (0 for empty)."""
        R, D = rows.shape
        key = torch.where(lid >= 0, lid, torch.full_like(lid, n_local))
        order = torch.argsort(key, stable=True)
        counts = torch.bincount(key, minlength=n_local + 1)
        offsets = torch.zeros(n_local + 1, dtype=torch.int32, device=rows.device)
        offsets[1:] = counts[:n_local].cumsum(0).to(torch.int32)
        xp = rows.index_select(0, order).contiguous()
        y = torch.zeros(R, D, dtype=rows.dtype, device=rows.device)
        if rows.is_cuda and rows.dtype == torch.bfloat16 and isinstance(L["experts_gate_up"][0], torch.Tensor):
            from .. import _native
            from ..models.moe import _stacked
            gu_w, down_w = _stacked(L)
            status = ops.ctx(rows.device).status
            gu = torch.empty(R, gu_w.shape[1], dtype=rows.dtype, device=rows.device)
            _native.C().grouped_gemm(xp, gu_w, offsets, gu, status)
            act = ops.silu_mul(gu).contiguous()
            yp = torch.empty(R, D, dtype=rows.dtype, device=rows.device)
            _native.C().grouped_gemm(act, down_w, offsets, yp, status)
            valid = (torch.arange(R, device=rows.device) < offsets[n_local])[:, None]
            y.index_copy_(0, order, torch.where(valid, yp, torch.zeros_like(yp)))
            return y
        off = offsets.tolist()  # CPU path: per-expert GEMMs
        for e in range(n_local):
            if off[e + 1] > off[e]:
                sel = order[off[e]:off[e + 1]]
                gu = ops.linear(rows.index_select(0, sel), L["experts_gate_up"][e])
                y.index_copy_(0, sel, ops.linear(ops.silu_mul(gu), L["experts_down"][e]))
        return y

    def forward_exact(self, model, layer_idx: int, L: dict, x: torch.Tensor, fb) -> torch.Tensor:
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
