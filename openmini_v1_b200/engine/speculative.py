"""Speculative decoding with an n-gram (prompt-lookup) proposer.

Each decode step proposes up to ``k`` draft tokens per sequence, by default by
matching the sequence's last n tokens (n = n_max .. n_min) against its earlier
history and copying what followed the most recent match. One forward over
[last token, draft_1 .. draft_m] per sequence (KV written for every row into
slots reserved ahead) gives the model's distribution after each prefix. KV of
rejected drafts sits in slots beyond the sequence length and is overwritten later.

* Greedy requests: the longest prefix of drafts equal to the model's argmax is
  accepted plus the model's next token, so a step emits 1 .. m+1 tokens and the
  output is identical to plain greedy decoding.
* Sampled requests (temperature > 0): speculative sampling with a deterministic
  draft (Leviathan, Kalman and Matias, "Fast inference from transformers via
  speculative decoding", ICML 2023; Chen et al., "Accelerating large language model
  decoding with speculative sampling", 2023). With the draft distribution a point
  mass on d_j, draft j is accepted with probability p_j(d_j), where p_j is the
  sampler's distribution at that row: temperature, then top-k, then top-p, the
  kept set of ``ops.reference.sample``. At the first rejection the token is drawn
  from p_j with d_j removed and renormalised; if every draft is accepted, a bonus
  token is drawn from p_m. The emitted sequence has exactly the sampler's
  distribution. The uniforms come from a generator keyed by (request seed, token
  offset), so a run repeats, but the stream differs from the non-speculative
  sampler's Philox stream.
* ``speculative_acceptance="typical"``: the typical-acceptance rule of Medusa (Cai et
  al., "Medusa: simple LLM inference acceleration framework with multiple decoding
  heads", 2024): draft j is accepted when p_j(d_j) > min(epsilon, delta exp(-H(p_j)))
  (H the entropy of p_j); at the first rejection the token is drawn from p_j. It
  accepts more drafts at high temperature but does not preserve the distribution.
* Adaptive draft length (per request): after a step with acceptance rate a/m >=
  ``speculative_accept_threshold`` the request's k grows by one, up to
  ``speculative_k_max``; below half the threshold it shrinks by one, down to
  ``speculative_k_min``.

Proposers: n-gram lookup, a draft model (``DraftModelProposer``) or a
multi-token-prediction head (``models.mtp.MTPProposer``, fed the hidden row
behind each sequence's last emitted token after every verified step).

Reference: draft / verify speculative decoding with adaptive draft length and
sampled acceptance (openmini-server/src/model/inference/speculative.rs:60-110,
503-560, speculative_decoding_v2.rs:22-57).
"""
from __future__ import annotations

import math
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
    return (p.repetition_penalty == 1.0 and not p.logprobs and not p.return_sampling_mask
            and not p.return_routing)


def _probs(row: torch.Tensor, p) -> torch.Tensor:
    """The sampler's distribution over one row of logits (fp32, on the row's device)."""
    from ..ops.reference import _cutoff_mask
    x = row.float() / p.temperature
    x = x - x.max()
    keep = _cutoff_mask(x, int(p.top_k), float(p.top_p))
    e = torch.where(keep, torch.exp(x), torch.zeros_like(x))
    return e / e.sum()


def _draw(prob: torch.Tensor, gen: torch.Generator) -> int:
    return int(torch.multinomial(prob.double().cpu(), 1, generator=gen))


def _seed(eng, r) -> int:
    return r.params.seed if r.params.seed is not None else eng.cfg.seed * 7919 + r.seq_id


def _verify_sampled(eng, r, dr: list, logits: torch.Tensor) -> list:
    """Speculative sampling of one request over its verify rows (logits [m + 1, V])."""
    gen = torch.Generator().manual_seed((_seed(eng, r) * 1000003 + r.rng_offset) & 0x7FFFFFFFFFFFFFFF)
    u = torch.rand(len(dr), generator=gen, dtype=torch.float64).tolist()
    cfg = eng.cfg
    typical = getattr(cfg, "speculative_acceptance", "exact") == "typical"
    if not typical and getattr(cfg, "speculative_acceptance", "exact") != "exact":
        raise ValueError(f"unknown speculative_acceptance {cfg.speculative_acceptance!r}")
    out = []
    for j, d in enumerate(dr):
        pj = _probs(logits[j], r.params)
        if typical:
            ent = float(-(pj * torch.log(pj.clamp(min=1e-30))).sum())
            if float(pj[d]) > min(cfg.typical_epsilon, cfg.typical_delta * math.exp(-ent)):
                out.append(d)
                continue
            out.append(_draw(pj, gen))
            return out
        if u[j] < float(pj[d]):
            out.append(d)
            continue
        pj[d] = 0.0
        out.append(_draw(pj / pj.sum(), gen))
        return out
    out.append(_draw(_probs(logits[len(dr)], r.params), gen))
    return out


def _adapt(eng, r, proposed: int, accepted: int):
    cfg = eng.cfg
    if not cfg.speculative_adaptive or proposed == 0:
        return
    k = getattr(r, "spec_k", cfg.speculative_k)
    rate = accepted / proposed
    if rate >= cfg.speculative_accept_threshold:
        k = min(k + 1, cfg.speculative_k_max or cfg.speculative_k)
    elif rate < cfg.speculative_accept_threshold / 2:
        k = max(k - 1, cfg.speculative_k_min)
    r.spec_k = k


def spec_decode_step(eng, so, proposer) -> list:
    """One verified speculative step for a pure decode batch (greedy and sampled requests)."""
    chunks = so.chunks
    rows_ids, rows_pos, rows_slot, rows_seq, rows_ctx = [], [], [], [], []
    drafts = []
    for si, c in enumerate(chunks):
        r = c.req
        p = r.num_tokens - 1
        room = min(getattr(r, "spec_k", proposer.k), r.params.max_tokens - len(r.output_token_ids) - 1,
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
    logits = eng.model.logits(x)
    greedy = logits.argmax(-1).to(torch.int32).cpu().tolist()
    observe = getattr(proposer, "observe", None)
    eng.stage.d2h_bytes = T * 4
    now = time.monotonic()
    outs = []
    o = 0
    eng.stats.setdefault("spec_proposed", 0)
    eng.stats.setdefault("spec_accepted", 0)
    for c, dr in zip(chunks, drafts):
        r = c.req
        if r.params.temperature > 0:
            new = _verify_sampled(eng, r, dr, logits[o:o + len(dr) + 1])
            a = len(new) - 1
        else:
            g = greedy[o:o + len(dr) + 1]
            a = 0
            while a < len(dr) and dr[a] == g[a]:
                a += 1
            new = dr[:a] + [g[a]]
        last_row = o + a  # hidden row whose prediction is the last emitted token
        o += len(dr) + 1
        eng.stats["spec_proposed"] += len(dr)
        eng.stats["spec_accepted"] += a
        _adapt(eng, r, len(dr), a)
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
            observe(r, x[last_row], new[-1])
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
