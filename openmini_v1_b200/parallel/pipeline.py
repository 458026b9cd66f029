"""Pipeline parallelism: a decoder split into stages, one stage per pipeline rank.

Stage ``p`` of ``P`` owns a contiguous layer range (layers split as evenly as
possible, earlier stages take the remainder). The first stage also owns the
embedding, the last the final RMSNorm and the LM head. Activations move
between stages with NCCL point-to-point send/recv (gloo on CPU) on the
pipeline group.

A forward pass is cut into ``microbatches`` contiguous row ranges. For each
microbatch a stage posts the receive of the *next* microbatch before it
computes the current one and sends its output with an asynchronous ``isend``,
so the transfer of microbatch i overlaps the compute of microbatch i+1 on both
sides of every stage boundary (GPipe-style fill, no bubbles inside a stage
beyond the first and last microbatch).

Every stage runs the same scheduler on the same requests (the ForwardBatch is
identical on all stages); the last stage's logits are what the engine samples
from, and ``broadcast_tokens`` hands the sampled tokens back to the other
stages so their schedulers stay in step.

Reference counterpart: ``ParallelStrategy::PipelineParallel`` and ``pp_degree``
(openmini-server/src/model/inference/distributed_inference_config.rs:54-60),
which the reference only logs (distributed_inference_engine.rs:350-352).
"""
from __future__ import annotations

import copy
from dataclasses import replace

import torch
import torch.distributed as dist

from .. import ops
from ..models.llama import DecoderLM, ForwardBatch


def stage_layers(num_layers: int, pp: int, stage: int) -> tuple[int, int]:
    """[l0, l1) of ``stage``: layers split evenly, the first ``num_layers % pp`` stages one more."""
    base, rem = divmod(num_layers, pp)
    l0 = stage * base + min(stage, rem)
    return l0, l0 + base + (1 if stage < rem else 0)


def split_rows(fb: ForwardBatch, parts: int) -> list:
    """Contiguous row ranges of ``fb`` as ForwardBatch views (block tables shared).

    Each part keeps the rows' cache slots, positions and visible-key counts, so
    attention over the paged cache is unchanged; prefill tiles are dropped (a
    part runs the row-wise paged attention kernel)."""
    T = fb.input_ids.shape[0]
    parts = max(1, min(parts, T))
    bounds = [T * i // parts for i in range(parts + 1)]
    out = []
    for a, b in zip(bounds[:-1], bounds[1:]):
        li = fb.logits_idx
        sel = (li >= a) & (li < b)
        out.append((a, b, replace(fb, input_ids=fb.input_ids[a:b], positions=fb.positions[a:b], slots=fb.slots[a:b],
                                  row_seq=fb.row_seq[a:b], row_ctx=fb.row_ctx[a:b], logits_idx=li[sel] - a,
                                  prefill_tiles=None, forced_routing=None, record_routing=None)))
    return out


class PipelineStage:
    """One pipeline stage of a decoder (wraps a DecoderLM holding only this stage's layers)."""

    def __init__(self, model: DecoderLM, par, layer_range: tuple[int, int], num_stages: int, stage: int):
        self.model = model
        self.par = par
        self.l0, self.l1 = layer_range
        self.pp = num_stages
        self.stage = stage
        self.first = stage == 0
        self.last = stage == num_stages - 1
        self.group = par.pp_group if par is not None else None

    # ------------------------------------------------------------------ construction
    @staticmethod
    def from_model(full: DecoderLM, par, num_stages: int, stage: int) -> "PipelineStage":
        """The stage's slice of an existing (full) model: shares its tensors."""
        l0, l1 = stage_layers(full.cfg.num_layers, num_stages, stage)
        cfg = copy.deepcopy(full.cfg)
        cfg.num_layers = l1 - l0
        m = DecoderLM(cfg, par=full.par, device=full.device, dtype=full.dtype, materialize=False,
                      weight_format=full.weight_format)
        m.layers = full.layers[l0:l1]
        m.embed, m.norm, m.lm_head = full.embed, full.norm, full.lm_head
        m._comm = full._comm
        return PipelineStage(m, par, (l0, l1), num_stages, stage)

    @staticmethod
    def random(cfg, par, device, seed: int = 0, weight_format: str = "bf16") -> "PipelineStage":
        """Random-init weights of this rank's stage only (the full model never exists)."""
        l0, l1 = stage_layers(cfg.num_layers, par.pp, par.pp_rank)
        scfg = copy.deepcopy(cfg)
        scfg.num_layers = l1 - l0
        m = DecoderLM(scfg, par=par, device=device, seed=seed * 131 + par.pp_rank, weight_format=weight_format)
        return PipelineStage(m, par, (l0, l1), par.pp, par.pp_rank)

    def allocate_kv(self, num_blocks: int):
        return self.model.allocate_kv(num_blocks)

    # ------------------------------------------------------------------ p2p
    def _peer(self, stage: int) -> int:
        return dist.get_global_rank(self.group, stage) if self.group is not None else stage

    def _irecv(self, rows: int):
        buf = torch.empty(rows, self.model.cfg.hidden_size, dtype=self.model.dtype, device=self.model.device)
        work = dist.irecv(buf, src=self._peer(self.stage - 1), group=self.group)
        return buf, work

    # ------------------------------------------------------------------ forward
    def forward(self, fb: ForwardBatch, kv, microbatches: int = 1):
        """Run this stage over ``fb``. Returns the last stage's final-normed hidden rows
        ``fb.logits_idx`` ([S', D]); other stages return None after sending their output."""
        m = self.model
        parts = split_rows(fb, microbatches) if microbatches > 1 else [(0, fb.input_ids.shape[0], fb)]
        pending = []  # outstanding isend works (and their buffers)
        outs = []
        nxt = self._irecv(parts[0][1] - parts[0][0]) if not self.first else None
        for i, (a, b, sub) in enumerate(parts):
            if self.first:
                h = m.embed_tokens(sub.input_ids)
            else:
                h, work = nxt
                work.wait()
                if i + 1 < len(parts):  # post the next receive before computing this one
                    nxt = self._irecv(parts[i + 1][1] - parts[i + 1][0])
            h = h.contiguous()
            delta = None
            for j, L in enumerate(m.layers):
                h, delta = m.layer_forward(j, L, h, delta, sub, kv)
            if delta is not None:
                h = h + delta
            if self.last:
                x = ops.rmsnorm(h, m.norm, m.cfg.rms_eps)
                outs.append(x.index_select(0, sub.logits_idx))
            else:
                pending.append((dist.isend(h, dst=self._peer(self.stage + 1), group=self.group), h))
        for w, _ in pending:
            w.wait()
        if not self.last:
            return None
        return torch.cat(outs) if len(outs) > 1 else outs[0]

    def logits(self, x):
        return self.model.logits(x) if x is not None else None

    def broadcast_tokens(self, tokens: torch.Tensor) -> torch.Tensor:
        """Sampled tokens from the last stage to every stage (in place)."""
        if self.pp > 1:
            dist.broadcast(tokens, src=self._peer(self.pp - 1), group=self.group)
        return tokens
