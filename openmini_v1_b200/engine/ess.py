"""Elastic storage: a two-tier cache for KV / latent-KV segments, device HBM first
and pinned host memory behind it, so contexts larger than the device budget stay
resident somewhere faster than recomputation.

* ``put(key, tensor)`` stores on the device tier; when the tier is over budget the
  eviction policy picks victims, which are demoted to the host tier (one
  ``copy_`` into a pinned buffer on a side stream) rather than dropped; the host
  tier in turn drops its own victims.
* ``get(key)`` returns the device tensor, promoting a host-resident entry first
  (a device miss on a host hit is counted separately from a full miss).
* Eviction policies: ``lru``, ``lfu``, and ``adaptive``, which keeps shadow lists
  of recently evicted keys for both and moves its weight towards whichever policy's
  victims are asked for again less often (the ARC idea of learning from ghost hits).
* A prefetcher watches the sequence of integer block ids asked for, recognises
  sequential / strided patterns and promotes the predicted next blocks ahead of use.

Reference counterpart: openmini-server/src/hardware/ess/{mod,cache,eviction,
prefetch,transfer}.rs (GPU/CPU tiers for the latent cache, LRU/LFU/adaptive
eviction, locality analyser and prefetcher; the reference stores byte vectors and
simulates the transfers; here the tiers hold real device and pinned host tensors).
"""
from __future__ import annotations

from collections import Counter, OrderedDict
from dataclasses import dataclass

import torch


@dataclass
class ESSStats:
    device_hits: int = 0
    host_hits: int = 0
    misses: int = 0
    demotions: int = 0
    promotions: int = 0
    drops: int = 0
    prefetches: int = 0


class _Policy:
    def __init__(self, kind: str):
        self.kind = kind
        self.lru: OrderedDict = OrderedDict()
        self.freq: Counter = Counter()
        self.ghost_lru: OrderedDict = OrderedDict()
        self.ghost_lfu: OrderedDict = OrderedDict()
        self.w_lru = 0.5

    def touch(self, key):
        self.lru[key] = None
        self.lru.move_to_end(key)
        self.freq[key] += 1
        if self.kind == "adaptive":  # a ghost hit says the other policy would have kept it
            if key in self.ghost_lru:
                self.w_lru = max(0.05, self.w_lru - 0.05)  # LRU evicted it too early
                del self.ghost_lru[key]
            if key in self.ghost_lfu:
                self.w_lru = min(0.95, self.w_lru + 0.05)
                del self.ghost_lfu[key]

    def forget(self, key):
        self.lru.pop(key, None)
        self.freq.pop(key, None)

    def victim(self, candidates):
        cands = [k for k in self.lru if k in candidates]
        if not cands:
            return None
        lru_v = cands[0]
        lfu_v = min(cands, key=lambda k: (self.freq[k], list(self.lru).index(k)))
        if self.kind == "lru":
            return lru_v
        if self.kind == "lfu":
            return lfu_v
        use_lru = self.w_lru >= 0.5
        v = lru_v if use_lru else lfu_v
        ghost = self.ghost_lru if use_lru else self.ghost_lfu
        ghost[v] = None
        while len(ghost) > 1024:
            ghost.popitem(last=False)
        return v


class StridePrefetcher:
    """Predicts the next ids from the last accesses: a constant stride seen ``confirm``
    times in a row gives ``depth`` predictions."""

    def __init__(self, depth: int = 2, confirm: int = 2):
        self.depth, self.confirm = depth, confirm
        self.hist: list[int] = []

    def access(self, addr: int) -> list[int]:
        self.hist = (self.hist + [addr])[-8:]
        if len(self.hist) < self.confirm + 1:
            return []
        d = [b - a for a, b in zip(self.hist[-self.confirm - 1:-1], self.hist[-self.confirm:])]
        if d[0] != 0 and all(x == d[0] for x in d):
            return [addr + d[0] * (i + 1) for i in range(self.depth)]
        return []

    def pattern(self) -> str:
        if len(self.hist) < 3:
            return "unknown"
        d = {b - a for a, b in zip(self.hist, self.hist[1:])}
        if d == {1}:
            return "sequential"
        if len(d) == 1:
            return "strided"
        return "random"


class ElasticStorage:
    def __init__(self, device_budget_bytes: int, host_budget_bytes: int, device="cpu", policy: str = "adaptive",
                 prefetch: bool = True):
        self.device = torch.device(device)
        self.dev_budget, self.host_budget = device_budget_bytes, host_budget_bytes
        self.dev: dict = {}
        self.host: dict = {}
        self.pol_dev = _Policy(policy)
        self.pol_host = _Policy("lru")
        self.prefetcher = StridePrefetcher() if prefetch else None
        self.stats = ESSStats()
        self._stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None

    @staticmethod
    def _nbytes(t: torch.Tensor) -> int:
        return t.numel() * t.element_size()

    def dev_used(self) -> int:
        return sum(self._nbytes(t) for t in self.dev.values())

    def host_used(self) -> int:
        return sum(self._nbytes(t) for t in self.host.values())

    # ------------------------------------------------------------------ tier moves
    def _to_host(self, t: torch.Tensor) -> torch.Tensor:
        if t.device.type != "cuda":
            return t.clone()
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        self._stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self._stream):
            h.copy_(t, non_blocking=True)
        self._stream.synchronize()
        return h

    def _to_device(self, h: torch.Tensor) -> torch.Tensor:
        return h.to(self.device, non_blocking=True) if self.device.type == "cuda" else h.clone()

    def _make_room_host(self, need: int):
        while self.host and self.host_used() + need > self.host_budget:
            v = self.pol_host.victim(self.host.keys())
            self.pol_host.forget(v)
            del self.host[v]
            self.stats.drops += 1

    def _make_room_dev(self, need: int, protect=()):
        while self.dev and self.dev_used() + need > self.dev_budget:
            v = self.pol_dev.victim([k for k in self.dev if k not in protect])
            if v is None:
                break
            t = self.dev.pop(v)
            self.pol_dev.forget(v)
            n = self._nbytes(t)
            if n <= self.host_budget:
                self._make_room_host(n)
                self.host[v] = self._to_host(t)
                self.pol_host.touch(v)
                self.stats.demotions += 1
            else:
                self.stats.drops += 1

    # ------------------------------------------------------------------ API
    def put(self, key, t: torch.Tensor):
        n = self._nbytes(t)
        if n > self.dev_budget and n > self.host_budget:
            raise ValueError(f"entry of {n} bytes is larger than either tier")
        self.remove(key)
        if n > self.dev_budget:  # too large for the device tier: host only
            self._make_room_host(n)
            self.host[key] = self._to_host(t)
            self.pol_host.touch(key)
            return
        self._make_room_dev(n, protect=(key,))
        self.dev[key] = t.to(self.device)
        self.pol_dev.touch(key)

    def _promote(self, key):
        h = self.host.pop(key)
        self.pol_host.forget(key)
        self._make_room_dev(self._nbytes(h), protect=(key,))
        self.dev[key] = self._to_device(h)
        self.pol_dev.touch(key)
        self.stats.promotions += 1

    def get(self, key):
        if key in self.dev:
            self.stats.device_hits += 1
            self.pol_dev.touch(key)
            out = self.dev[key]
        elif key in self.host:
            self.stats.host_hits += 1
            if self._nbytes(self.host[key]) > self.dev_budget:
                # larger than the device tier: served as a temporary device copy, kept on the host
                self.pol_host.touch(key)
                out = self._to_device(self.host[key])
            else:
                self._promote(key)
                out = self.dev[key]
        else:
            self.stats.misses += 1
            out = None
        if self.prefetcher is not None and isinstance(key, int):
            for p in self.prefetcher.access(key):
                if p in self.host and self._nbytes(self.host[p]) <= self.dev_budget:
                    self._promote(p)
                    self.stats.prefetches += 1
        return out

    def tier(self, key) -> str | None:
        return "device" if key in self.dev else "host" if key in self.host else None

    def remove(self, key):
        for tier, pol in ((self.dev, self.pol_dev), (self.host, self.pol_host)):
            if key in tier:
                del tier[key]
                pol.forget(key)

    def clear(self):
        for k in list(self.dev) + list(self.host):
            self.remove(k)
