"""Speculative decoding with an n-gram (prompt-lookup) proposer.

For greedy requests, each decode step proposes up to ``k`` draft tokens per
sequence by matching the sequence's last n tokens (n = n_max .. n_min) against
its earlier history and copying what followed the most recent match. One
forward over [last token, draft_1 .. draft_m] per sequence (KV written for
every row into slots reserved ahead) yields the model's greedy choice after
each prefix; the longest prefix of drafts equal to those choices is accepted
plus the model's next token, so a step emits 1 .. m+1 tokens and the output
is identical to plain greedy decoding. KV of rejected drafts sits in slots
beyond the sequence length and is overwritten later.

Proposers: n-gram lookup, a draft model (``DraftModelProposer``) or a
multi-token-prediction head (``models.mtp.MTPProposer``, fed the hidden row
behind each sequence's last emitted token after every verified step).

Reference: draft / verify speculative decoding with adaptive k
(openmini-server/src/model/inference/speculative.rs,
speculative_decoding_v2.rs); the proposer here needs no draft model.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from ..models.llama import ForwardBatch
from .request import RequestOutput


class NgramProposer:
    def __init__(self, k: int = 4, n_max: int = 3, n_min: int = 1):
        self.k, self.n_max, self.n_min = k, n_max, n_min

    def propose(self, toks, k: int | None = None) -> list:
        k = self.k if k is None else k
        L = len(toks)
        if k <= 0 or L < 2:
            return []
        arr = np.asarray(toks, dtype=np.int64)
        for n in range(min(self.n_max, L - 1), self.n_min - 1, -1):
            pat = arr[L - n:]
            # most recent earlier occurrence of the last n tokens
            win = np.lib.stride_tricks.sliding_window_view(arr[:L - 1], n)
            hits = np.nonzero((win == pat).all(axis=1))[0]
            if hits.size:
                s = int(hits[-1]) + n
                return arr[s:s + k].tolist()
        return []


class DraftModelProposer:
    """Draft-model proposer (the reference's draft / verify scheme): a smaller model of the
    same vocabulary runs greedily for k tokens from the sequence so far. It serves from
    its own engine with the prefix cache on, so consecutive proposals for one sequence
    re-use the draft KV of the shared prefix and cost about k draft decode steps."""

    def __init__(self, draft_engine, k: int = 4):
        from .request import SamplingParams
        self.eng, self.k = draft_engine, k
        self._sp = SamplingParams

    def propose(self, toks, k: int | None = None) -> list:
        k = self.k if k is None else k
        if k <= 0:
            return []
        r = self.eng.generate([list(toks)], self._sp(temperature=0.0, max_tokens=k, ignore_eos=True))[0]
        return list(r.output_token_ids)


def eligible(r) -> bool:
    p = r.params
    return (p.temperature == 0.0 and p.repetition_penalty == 1.0 and not p.logprobs and not p.return_sampling_mask
            and not p.return_routing)


def spec_decode_step(eng, so, proposer) -> list:
    """One verified speculative step for a pure decode batch of greedy requests."""
    chunks = so.chunks
    rows_ids, rows_pos, rows_slot, rows_seq, rows_ctx = [], [], [], [], []
    drafts = []
    for si, c in enumerate(chunks):
        r = c.req
        p = r.num_tokens - 1
        room = min(proposer.k, r.params.max_tokens - len(r.output_token_ids) - 1,
                   eng.cfg.max_model_len - r.num_tokens - 1)
        if getattr(proposer, "wants_request", False):
            d = proposer.propose(r.all_token_ids, max(room, 0), req=r)
        else:
            d = proposer.propose(r.all_token_ids, max(room, 0))
        if d:
            try:
                eng.bm.reserve(r.seq_id, len(d) + 1)
            except RuntimeError:
                d = []
        toks = [r.all_token_ids[-1]] + d
        drafts.append(d)
        rows_ids += toks
        rows_pos += range(p, p + len(toks))
        rows_slot += eng.bm.slots(r.seq_id, p, p + len(toks))
        rows_seq += [si] * len(toks)
        rows_ctx += range(p + 1, p + len(toks) + 1)
    T, S, mb = len(rows_ids), len(chunks), eng.max_blocks_per_seq
    bt = np.zeros((S, mb), dtype=np.int32)
    eng.bm.fill_block_tables([c.req.seq_id for c in chunks], bt)
    dev = eng.device
    i32 = dict(dtype=torch.int32)
    host = torch.tensor(np.concatenate([np.asarray(x, dtype=np.int32) for x in
                                        (rows_ids, rows_pos, rows_slot, rows_seq, rows_ctx)]), **i32)
    d = host.to(dev, non_blocking=True)
    fb = ForwardBatch(input_ids=d[0:T], positions=d[T:2 * T], slots=d[2 * T:3 * T], row_seq=d[3 * T:4 * T],
                      row_ctx=d[4 * T:5 * T], block_tables=torch.from_numpy(bt).to(dev),
                      max_ctx=eng.cfg.max_model_len, logits_idx=torch.arange(T, device=dev))
    eng.stage.h2d_bytes = host.numel() * 4 + bt.size * 4
    x = eng.model(fb, eng.kv)
    greedy = eng.model.logits(x).argmax(-1).to(torch.int32).cpu().tolist()
    observe = getattr(proposer, "observe", None)
    eng.stage.d2h_bytes = T * 4
    now = time.monotonic()
    outs = []
    o = 0
    eng.stats.setdefault("spec_proposed", 0)
    eng.stats.setdefault("spec_accepted", 0)
    for c, dr in zip(chunks, drafts):
        r = c.req
        g = greedy[o:o + len(dr) + 1]
        a = 0
        while a < len(dr) and dr[a] == g[a]:
            a += 1
        new = dr[:a] + [g[a]]
        last_row = o + a  # hidden row whose prediction is the last emitted token
        o += len(dr) + 1
        eng.stats["spec_proposed"] += len(dr)
        eng.stats["spec_accepted"] += a
        r.num_computed = r.num_tokens
        emitted, reason = [], None
        for t in new:
            r.output_token_ids.append(int(t))
            r.rng_offset += 1
            emitted.append(int(t))
            eng.stats["decode_tokens"] += 1
            if r.first_token_time is None:
                r.first_token_time = now
            reason = eng._stop_reason(r, int(t))
            if reason:
                break
        if observe is not None and not reason:
            observe(r, x[last_row], g[a])
        if reason:
            r.finish_reason, r.finish_time = reason, now
            eng.sched.finish(r)
            eng.requests.pop(r.request_id, None)
            if hasattr(proposer, "forget"):
                proposer.forget(r)
        outs.append(RequestOutput(request_id=r.request_id, new_token_ids=emitted,
                                  output_token_ids=r.output_token_ids, finished=reason is not None,
                                  finish_reason=reason, prompt_tokens=len(r.prompt_token_ids)))
    return outs
