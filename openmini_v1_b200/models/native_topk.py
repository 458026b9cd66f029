"""Heuristic key selection for sparse attention ("native top-k").

Given queries q [T, d] and keys k [S, d] (the last T of the S positions are the
queries' own, so query i may see keys j <= i + S - T when ``causal``), returns for
every query row the indices of at most ``top_k`` keys to attend to, [T, top_k]
int64 with -1 padding, best first by the score q . k. Modes:

* ``"exact"``: the top_k keys by score (the DSA indexer's selection rule).
* ``"query_norm"``: rows whose query norm is at least ``norm_ratio`` x the largest
  norm in the batch (high-activation queries) get the exact selection; the others
  choose among a local window of floor(sqrt(S)) keys ending at their own position
  plus an evenly strided sample of the visible keys (a quarter of the budget).
* ``"key_similarity"``: keys are grouped greedily into clusters of cosine similarity
  >= ``sim_threshold`` to the cluster's first key; each query ranks the clusters by
  the score of their first key and takes the best max(1, top_k / clusters) keys of
  each cluster in that order until top_k are chosen.
* ``"combined"`` (default): the union of the exact top (top_k x ``candidate_multiplier``
  / 2) and of the keys most similar to the key at the query's own position (the same
  count) is re-ranked by score.

Every mode returns only visible keys, each at most once; with top_k >= the number of
visible keys every mode returns all of them.

Reference counterpart: the Native Top-K engine of
openmini-server/src/model/inference/native_top_k.rs:84-99 (constants), 128-135
(modes), 567-700 and 765-960 (selection).
"""
from __future__ import annotations

import math

import torch

MODES = ("exact", "query_norm", "key_similarity", "combined")


def _visible(T: int, S: int, causal: bool, device) -> torch.Tensor:
    if not causal:
        return torch.ones(T, S, dtype=torch.bool, device=device)
    return torch.arange(S, device=device)[None, :] <= torch.arange(T, device=device)[:, None] + (S - T)


def _take(scores: torch.Tensor, allowed: torch.Tensor, top_k: int) -> torch.Tensor:
    s = torch.where(allowed, scores, torch.full_like(scores, -math.inf))
    kk = min(top_k, s.shape[1])
    v, idx = torch.topk(s, kk, dim=1)
    idx = torch.where(torch.isfinite(v), idx, torch.full_like(idx, -1))
    if kk < top_k:
        idx = torch.cat([idx, idx.new_full((idx.shape[0], top_k - kk), -1)], 1)
    return idx


def clusters_by_similarity(k: torch.Tensor, threshold: float) -> torch.Tensor:
    """Greedy clustering: key j joins the most similar existing cluster head when the
    cosine similarity is >= threshold, else it starts a cluster. Returns the cluster id
    of every key [S] (ids in order of first appearance)."""
    kn = torch.nn.functional.normalize(k.float(), dim=-1)
    heads = []
    cid = torch.empty(k.shape[0], dtype=torch.long, device=k.device)
    for j in range(k.shape[0]):
        if heads:
            sim = kn[heads] @ kn[j]
            best = int(torch.argmax(sim))
            if float(sim[best]) >= threshold:
                cid[j] = best
                continue
        cid[j] = len(heads)
        heads.append(j)
    return cid


def native_topk(q: torch.Tensor, k: torch.Tensor, top_k: int, mode: str = "combined", causal: bool = True,
                norm_ratio: float = 0.7, sim_threshold: float = 0.85, candidate_multiplier: int = 4) -> torch.Tensor:
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}")
    T, S = q.shape[0], k.shape[0]
    scores = q.float() @ k.float().t()
    vis = _visible(T, S, causal, q.device)
    if mode == "exact":
        return _take(scores, vis, top_k)
    if mode == "query_norm":
        norms = q.float().norm(dim=-1)
        hi = norms >= norm_ratio * norms.max()
        w = max(1, int(math.isqrt(S)))
        pos = torch.arange(T, device=q.device)[:, None] + (S - T)
        j = torch.arange(S, device=q.device)[None, :]
        local = (j > pos - w) & (j <= pos)
        step = max(1, S // max(1, top_k - (3 * top_k) // 4))
        strided = (j % step) == 0
        allowed = torch.where(hi[:, None], vis, vis & (local | strided))
        # rows left with fewer candidates than their budget take their most recent keys too
        need = torch.minimum(vis.sum(1), torch.tensor(top_k, device=q.device))
        short = allowed.sum(1) < need
        allowed |= short[:, None] & vis & (pos - j < need[:, None])
        return _take(scores, allowed, top_k)
    if mode == "key_similarity":
        cid = clusters_by_similarity(k, sim_threshold)
        C = int(cid.max()) + 1
        heads = torch.stack([torch.nonzero(cid == c)[0, 0] for c in range(C)])
        per = max(1, top_k // C)
        out = torch.full((T, top_k), -1, dtype=torch.long, device=q.device)
        for i in range(T):
            vi = vis[i]
            order = torch.argsort(scores[i, heads], descending=True)
            chosen = []
            for c in order.tolist():
                members = torch.nonzero((cid == c) & vi).flatten()
                if members.numel() == 0:
                    continue
                best = members[torch.argsort(scores[i, members], descending=True)[:per]]
                chosen.extend(best.tolist())
                if len(chosen) >= top_k:
                    break
            if len(chosen) < min(top_k, int(vi.sum())):  # fill from the best remaining visible keys
                rest = vi.clone()
                rest[chosen] = False
                extra = _take(scores[i:i + 1], rest[None], top_k - len(chosen))[0]
                chosen.extend(x for x in extra.tolist() if x >= 0)
            chosen = torch.tensor(chosen[:top_k], dtype=torch.long, device=q.device)
            chosen = chosen[torch.argsort(scores[i, chosen], descending=True)]
            out[i, :chosen.numel()] = chosen
        return out
    half = max(1, top_k * candidate_multiplier // 2)
    cand = torch.zeros(T, S, device=q.device)
    kn = torch.nn.functional.normalize(k.float(), dim=-1)
    own = kn[(torch.arange(T, device=q.device) + (S - T)).clamp(0, S - 1)]
    for idx in (_take(scores, vis, half), _take(own @ kn.t(), vis, half)):
        # amax: a padding entry (-1, written at column 0 with value 0) never clears a chosen key
        cand.scatter_reduce_(1, idx.clamp(min=0), (idx >= 0).float(), reduce="amax")
    return _take(scores, (cand > 0) & vis, top_k)
