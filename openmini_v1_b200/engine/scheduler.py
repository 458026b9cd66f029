"""Continuous-batching scheduler.

Behaviour of the reference BatchScheduler
(openmini-server/src/hardware/kv_cache/continuous_batch.rs:17-480): a waiting
queue feeding a bounded running set, KV-block reservation before admission,
preemption of the least important request when the cache runs out, TTFT
bookkeeping. Differences: prompts may be prefilled in chunks under a token
budget, prefix-cache hits skip recomputation, and preemption is by recompute
(blocks freed, request re-queued at the front).

Each ``schedule()`` returns either a prefill batch (prompt chunks) or a decode
batch (one token for every running request) so decode steps have a fixed
shape that CUDA graphs can replay.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

from .request import Request, RequestStatus


@dataclass
class ScheduledChunk:
    req: Request
    start: int        # first token position computed in this step
    end: int          # one past the last
    wants_logits: bool


@dataclass
class SchedulerOutput:
    kind: str                          # "prefill" | "decode" | "idle"
    chunks: list = field(default_factory=list)
    preempted: list = field(default_factory=list)

    @property
    def num_tokens(self):
        return sum(c.end - c.start for c in self.chunks)


class Scheduler:
    def __init__(self, block_manager, max_num_seqs=256, max_num_batched_tokens=8192, max_model_len=8192,
                 enable_chunked_prefill=True):
        self.bm = block_manager
        self.max_num_seqs = max_num_seqs
        self.max_batched = max_num_batched_tokens
        self.max_model_len = max_model_len
        self.chunked = enable_chunked_prefill
        self.waiting: deque = deque()
        self.running: list = []
        self.swapper = None  # KVSwapper: preempt by swapping KV to host instead of recompute

    # ------------------------------------------------------------ queue ops
    def add(self, req: Request):
        if len(req.prompt_token_ids) == 0:
            raise ValueError("empty prompt")
        if len(req.prompt_token_ids) + req.params.max_tokens > self.max_model_len:
            raise ValueError(f"prompt + max_tokens exceeds max_model_len={self.max_model_len}")
        req.status = RequestStatus.WAITING
        self.waiting.append(req)

    def abort(self, request_id: str):
        for q in (self.waiting, self.running):
            for r in list(q):
                if r.request_id == request_id:
                    q.remove(r)
                    self.bm.free(r.seq_id)
                    r.status = RequestStatus.ABORTED
                    return r
        return None

    def finish(self, req: Request):
        if req in self.running:
            self.running.remove(req)
        self.bm.free(req.seq_id)
        req.status = RequestStatus.FINISHED

    def has_unfinished(self):
        return bool(self.waiting or self.running)

    # ------------------------------------------------------------ policy
    def _victim(self, exclude):
        cands = [r for r in self.running if r is not exclude]
        if not cands:
            return None
        return max(cands, key=lambda r: (r.priority, r.arrival))

    def _preempt(self, r: Request, out: SchedulerOutput):
        self.running.remove(r)
        if self.swapper is not None:
            self.swapper.swap_out(r)  # KV of the computed prefix kept on the host
        else:
            r.routing = {}  # recomputed from scratch on re-admission
        self.bm.free(r.seq_id)
        r.num_computed = 0
        r.num_preemptions += 1
        r.status = RequestStatus.WAITING
        self.waiting.appendleft(r)
        out.preempted.append(r)

    def schedule(self) -> SchedulerOutput:
        out = SchedulerOutput(kind="idle")
        budget = self.max_batched
        # 1) continue partially prefilled running requests first
        for r in [r for r in self.running if r.in_prefill]:
            if budget <= 0:
                break
            n = min(r.num_tokens - r.num_computed, budget)
            out.chunks.append(ScheduledChunk(r, r.num_computed, r.num_computed + n,
                                             r.num_computed + n == r.num_tokens))
            budget -= n
        # 2) admit waiting requests
        while self.waiting and budget > 0 and len(self.running) < self.max_num_seqs:
            r = self.waiting[0]
            toks = r.all_token_ids
            if not self.bm.can_allocate(len(toks) + 1):
                break
            if not self.chunked and len(toks) > budget and out.chunks:
                break
            self.waiting.popleft()
            cached = self.bm.allocate(r.seq_id, toks)
            if getattr(r, "swapped", None) and self.swapper is not None:
                n_sw = r.swapped[0]
                if self.bm.seq_len(r.seq_id) >= n_sw:
                    cached = max(cached, self.swapper.swap_in(r))
            cached = min(cached, len(toks) - 1)  # the last token is always run (its logits are needed)
            r.num_computed = cached
            r.status = RequestStatus.RUNNING
            self.running.append(r)
            n = len(toks) - cached
            if self.chunked:
                n = min(n, budget)
            out.chunks.append(ScheduledChunk(r, cached, cached + n, cached + n == len(toks)))
            budget -= n
        if out.chunks:
            out.kind = "prefill"
            return out
        # 3) decode every running request (one token each)
        decode = [r for r in self.running if not r.in_prefill]
        gone = set()  # preempted this step (requests hash by identity)
        held = {}     # request -> free blocks its append this step takes (reserved cumulatively)
        used = 0      # sum of held
        free = self.bm.num_free()
        for r in decode:
            if r in gone:
                continue
            need = self.bm.append_need(r.seq_id, 1)
            if need > free - used:
                while need > free - used:
                    v = self._victim(r)
                    if v is None:
                        break
                    self._preempt(v, out)
                    gone.add(v)
                    used -= held.pop(v, 0)
                    free = self.bm.num_free()
                if need > free - used:
                    self._preempt(r, out)
                    gone.add(r)
                    free = self.bm.num_free()
                    continue
            held[r] = need
            used += need
        if gone:
            decode = [r for r in decode if r not in gone]
        for r in decode:
            pos = r.num_tokens - 1
            out.chunks.append(ScheduledChunk(r, pos, pos + 1, True))
        out.kind = "decode" if out.chunks else "idle"
        return out
