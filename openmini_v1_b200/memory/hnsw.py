"""Hierarchical navigable small-world graph index (Malkov and Yashunin, 2016) for
cosine similarity over unit vectors.

Nodes get a top level drawn from floor(-ln(U) / ln(M)); insertion descends greedily
from the entry point to the node's top level, then on every level below runs a
best-first search with ``ef_construction`` candidates and links the node to its M
nearest (2 M on level 0), pruning neighbours that exceed the degree bound. Queries
descend greedily and finish with a best-first search of width ``ef`` on level 0.

Reference counterpart: openmini-server/src/model/inference/memory/hnsw.rs.
"""
from __future__ import annotations

import heapq
import math
import random

import numpy as np


class HNSWIndex:
    def __init__(self, dim: int, M: int = 16, ef_construction: int = 100, ef: int = 64, seed: int = 0):
        self.dim, self.M, self.efc, self.ef = dim, M, ef_construction, ef
        self.mL = 1.0 / math.log(M)
        self.rng = random.Random(seed)
        self.vecs = np.zeros((0, dim), dtype=np.float32)
        self.levels: list[int] = []
        self.links: list[list[list[int]]] = []   # node -> level -> neighbours
        self.entry = -1
        self.top = -1

    def __len__(self):
        return len(self.levels)

    @staticmethod
    def _unit(v):
        v = np.asarray(v, dtype=np.float32)
        n = np.linalg.norm(v, axis=-1, keepdims=True)
        return v / np.where(n > 0, n, 1)

    def _dist(self, q, ids):
        return 1.0 - self.vecs[ids] @ q

    def _search_layer(self, q, entries, ef, level):
        visited = set(entries)
        d0 = self._dist(q, list(entries))
        cand = [(float(d), e) for d, e in zip(d0, entries)]
        heapq.heapify(cand)
        best = [(-d, e) for d, e in cand]
        heapq.heapify(best)
        while len(best) > ef:
            heapq.heappop(best)
        while cand:
            d, c = heapq.heappop(cand)
            if d > -best[0][0] and len(best) >= ef:
                break
            nb = [n for n in self.links[c][level] if n not in visited]
            if not nb:
                continue
            visited.update(nb)
            for dn, n in zip(self._dist(q, nb), nb):
                dn = float(dn)
                if len(best) < ef or dn < -best[0][0]:
                    heapq.heappush(cand, (dn, n))
                    heapq.heappush(best, (-dn, n))
                    if len(best) > ef:
                        heapq.heappop(best)
        return sorted((-d, e) for d, e in best)

    def add(self, v) -> int:
        q = self._unit(v).reshape(self.dim)
        i = len(self.levels)
        self.vecs = np.vstack([self.vecs, q[None]])
        lvl = int(-math.log(max(self.rng.random(), 1e-12)) * self.mL)
        self.levels.append(lvl)
        self.links.append([[] for _ in range(lvl + 1)])
        if self.entry < 0:
            self.entry, self.top = i, lvl
            return i
        ep = [self.entry]
        for L in range(self.top, lvl, -1):
            ep = [self._search_layer(q, ep, 1, L)[0][1]]
        for L in range(min(lvl, self.top), -1, -1):
            res = self._search_layer(q, ep, self.efc, L)
            mmax = 2 * self.M if L == 0 else self.M
            nbrs = [e for _, e in res[: self.M]]
            self.links[i][L] = nbrs
            for n in nbrs:
                ln = self.links[n][L]
                ln.append(i)
                if len(ln) > mmax:  # keep the closest
                    d = self._dist(self.vecs[n], ln)
                    self.links[n][L] = [ln[j] for j in np.argsort(d)[:mmax]]
            ep = [e for _, e in res]
        if lvl > self.top:
            self.entry, self.top = i, lvl
        return i

    def search(self, v, k: int = 10, ef: int | None = None):
        """-> [(cosine similarity, id)] best first."""
        if self.entry < 0:
            return []
        q = self._unit(v).reshape(self.dim)
        ep = [self.entry]
        for L in range(self.top, 0, -1):
            ep = [self._search_layer(q, ep, 1, L)[0][1]]
        res = self._search_layer(q, ep, max(ef or self.ef, k), 0)
        return [(1.0 - d, e) for d, e in res[:k]]

    def state(self) -> dict:
        return {"dim": self.dim, "M": self.M, "efc": self.efc, "ef": self.ef, "vecs": self.vecs,
                "levels": self.levels, "links": self.links, "entry": self.entry, "top": self.top}

    @classmethod
    def from_state(cls, s: dict) -> "HNSWIndex":
        ix = cls(s["dim"], s["M"], s["efc"], s["ef"])
        ix.vecs, ix.levels, ix.links, ix.entry, ix.top = s["vecs"], s["levels"], s["links"], s["entry"], s["top"]
        return ix
