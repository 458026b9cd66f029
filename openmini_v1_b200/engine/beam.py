"""Beam search over the paged KV cache (fork + copy-on-write blocks).

Reference: the sampler's beam search (openmini-server/src/model/inference/sampler.rs:452-560):
keep the ``beam_width`` best partial sequences by summed log-probability,
extend each by its best tokens, rank finished hypotheses by length-normalised
score ``sum_logp / len**length_penalty``.

Here every beam is a sequence of the engine's block manager. The prompt is
prefilled once; a beam that is extended by k tokens is forked k-1 times
(``BlockManager.fork`` shares all blocks by reference count) and the first
append into a shared partial block copies it (copy-on-write, applied on the
device by ``LLMEngine._apply_cow``). One decode forward per step runs all live
beams as one batch through the same model and attention kernels as sampling.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .request import Request, SamplingParams
from .scheduler import ScheduledChunk, SchedulerOutput


@dataclass
class Hypothesis:
    token_ids: list
    logprob: float
    finished: bool

    def score(self, length_penalty: float) -> float:
        return self.logprob / max(1, len(self.token_ids)) ** length_penalty


def beam_search(engine, prompt_token_ids, beam_width: int = 4, max_tokens: int = 32, length_penalty: float = 1.0,
                eos_token_id: int | None = None) -> list:
    """Returns the finished hypotheses, best first (at most ``beam_width``)."""
    if engine.has_unfinished():
        raise RuntimeError("beam search needs an idle engine (it uses the KV cache directly)")
    bm = engine.bm
    sp = SamplingParams(temperature=0.0, max_tokens=max_tokens)
    root = Request("beam-0", list(prompt_token_ids), sp)
    if not bm.can_allocate(len(root.prompt_token_ids) + beam_width * (max_tokens + 16)):
        raise RuntimeError("not enough KV blocks for the beams")
    bm.allocate(root.seq_id, root.prompt_token_ids)
    live = [(root, 0.0)]
    done: list = []
    n_fork = 0
    try:
        so = SchedulerOutput("prefill", [ScheduledChunk(root, 0, len(root.prompt_token_ids), True)])
        for step in range(max_tokens):
            fb, _, rows = engine._build(so)
            logits = engine.model.logits(engine.model(fb, engine.kv)).float()
            logp = torch.log_softmax(logits, dim=-1).cpu()
            cands = []
            for i, (r, s) in enumerate(live):
                top = torch.topk(logp[i], beam_width)
                for lp, t in zip(top.values.tolist(), top.indices.tolist()):
                    cands.append((s + lp, i, t))
            cands.sort(key=lambda c: -c[0])
            new_live = []
            used = {}
            for score, i, t in cands:
                parent = live[i][0]
                toks = parent.output_token_ids + [t]
                if (eos_token_id is not None and t == eos_token_id) or len(toks) >= max_tokens:
                    done.append(Hypothesis(toks, score, True))
                    if len(done) >= beam_width and len(new_live) == 0:
                        break
                    continue
                if len(new_live) >= beam_width:
                    continue
                if i not in used:  # first child reuses the parent's sequence
                    child = parent
                    used[i] = 0
                else:
                    n_fork += 1
                    child = Request(f"beam-{n_fork}", list(parent.prompt_token_ids), sp)
                    child.output_token_ids = list(parent.output_token_ids)
                    bm.fork(parent.seq_id, child.seq_id)
                    used[i] += 1
                new_live.append((child, score, t))
            # parents that produced no live child release their blocks
            keep = {id(c) for c, _, _ in new_live}
            for r, _ in live:
                if id(r) not in keep:
                    bm.free(r.seq_id)
            if not new_live or (len(done) >= beam_width and
                                max(s for _, s, _ in new_live) <= max(h.logprob for h in done)):
                for c, _, _ in new_live:
                    bm.free(c.seq_id)
                live = []
                break
            live = []
            chunks = []
            for c, s, t in new_live:
                c.output_token_ids.append(t)
                engine._apply_cow(bm.append(c.seq_id, [t]))
                pos = c.num_tokens - 1
                chunks.append(ScheduledChunk(c, pos, pos + 1, True))
                live.append((c, s))
            so = SchedulerOutput("decode", chunks)
        for r, s in live:  # ran out of steps
            done.append(Hypothesis(list(r.output_token_ids), s, False))
            bm.free(r.seq_id)
    except BaseException:
        for r, _ in live:
            bm.free(r.seq_id)
        raise
    done.sort(key=lambda h: -h.score(length_penalty))
    return done[:beam_width]
