"""Rollout-state replay for RL training.

Keep Routing (openmini-server/src/rl/keep_routing.rs:14-180): the expert ids
each MoE layer chose for each token during the rollout are stored and forced
in the training forward, so the policy gradient is taken through the experts
that actually produced the sample (Strict mode), or the stored routing is used
only where it still exists (Soft), or not at all (None).

Keep Sampling Mask (openmini-server/src/rl/keep_sampling_mask.rs:10-185): the
top-k / top-p kept set of every sampled token (a bitmask over the vocabulary
written by the device sampler) is stored and re-applied to the training
logits, so log-probabilities are computed under the truncated distribution the
token was actually drawn from.

Both caches are bounded (oldest entries evicted) and keyed by sample id.
"""
from __future__ import annotations

import enum
import threading
from collections import OrderedDict

import torch


class EnforceMode(enum.Enum):
    STRICT = "strict"
    SOFT = "soft"
    NONE = "none"


class _LRU:
    def __init__(self, max_items: int):
        self.max = max_items
        self.d = OrderedDict()
        self.lock = threading.Lock()

    def put(self, k, v):
        with self.lock:
            self.d[k] = v
            self.d.move_to_end(k)
            while len(self.d) > self.max:
                self.d.popitem(last=False)

    def get(self, k):
        with self.lock:
            v = self.d.get(k)
            if v is not None:
                self.d.move_to_end(k)
            return v

    def pop(self, k):
        with self.lock:
            return self.d.pop(k, None)

    def clear(self):
        with self.lock:
            self.d.clear()

    def __len__(self):
        return len(self.d)

    def save_file(self, path: str):
        """Write the entries (oldest first) with torch.save; a rollout worker's caches
        can then be replayed by a trainer in another process."""
        with self.lock:
            items = list(self.d.items())
        torch.save({"format": "openmini-replay-cache", "version": 1, "items": items}, path)

    def load_file(self, path: str) -> int:
        """Add the entries of a file written by ``save_file``; returns how many."""
        blob = torch.load(path, map_location="cpu", weights_only=True)
        if blob.get("format") != "openmini-replay-cache":
            raise ValueError(f"{path} is not a replay cache file")
        for k, v in blob["items"]:
            self.put(k, v)
        return len(blob["items"])


class KeepRouting:
    """Per-sample router decisions: {layer: expert ids int32 [T, k]}."""

    def __init__(self, max_caches: int = 1000, mode: EnforceMode = EnforceMode.STRICT):
        self.cache = _LRU(max_caches)
        self.mode = mode

    def save_routing(self, key: str, routing: dict):
        self.cache.put(key, {int(l): ids.detach().to("cpu", torch.int32) for l, ids in routing.items()})

    def get_routing(self, key: str):
        return self.cache.get(key)

    def apply_routing(self, key: str, device=None, n_tokens: int | None = None):
        """Forced routing for the training forward, or None (route freely)."""
        if self.mode == EnforceMode.NONE:
            return None
        r = self.cache.get(key)
        if r is None:
            if self.mode == EnforceMode.STRICT:
                raise KeyError(f"no stored routing for {key!r} (strict Keep Routing)")
            return None
        if n_tokens is not None and any(v.shape[0] != n_tokens for v in r.values()):
            if self.mode == EnforceMode.STRICT:
                raise ValueError("stored routing does not match the token count")
            return None
        return {l: v.to(device) for l, v in r.items()}

    def clear(self):
        self.cache.clear()

    def save_file(self, path: str):
        self.cache.save_file(path)

    def load_file(self, path: str) -> int:
        return self.cache.load_file(path)


class KeepSamplingMask:
    """Per-sample kept sets: packed int32 bit words [n_sampled, ceil(V/32)] and valid lengths."""

    def __init__(self, max_masks: int = 1000):
        self.cache = _LRU(max_masks)

    def save(self, key: str, words: torch.Tensor, valid_length: int | None = None):
        self.cache.put(key, (words.detach().to("cpu", torch.int32), valid_length or words.shape[0]))

    def get(self, key: str):
        return self.cache.get(key)

    def apply(self, key: str, logits: torch.Tensor) -> torch.Tensor:
        """Set logits outside the stored kept set to -inf (rows beyond the stored length untouched)."""
        item = self.cache.get(key)
        if item is None:
            return logits
        words, n = item
        return apply_mask_words(logits, words[:n].to(logits.device))

    def clear(self):
        self.cache.clear()

    def save_file(self, path: str):
        self.cache.save_file(path)

    def load_file(self, path: str) -> int:
        return self.cache.load_file(path)


def unpack_words(words: torch.Tensor, V: int) -> torch.Tensor:
    w = words.to(torch.int64) & 0xFFFFFFFF
    bits = (w[:, :, None] >> torch.arange(32, device=words.device)) & 1
    return bits.reshape(words.shape[0], -1)[:, :V].bool()


def apply_mask_words(logits: torch.Tensor, words: torch.Tensor) -> torch.Tensor:
    n, V = min(words.shape[0], logits.shape[0]), logits.shape[-1]
    keep = unpack_words(words[:n], V)
    out = logits.clone()
    out[:n] = logits[:n].masked_fill(~keep, float("-inf"))
    return out


def merge_masks(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Product (intersection) of two packed kept sets."""
    return a & b


def termination_mask(lengths, max_len: int) -> torch.Tensor:
    """[B, max_len] bool, True for positions before each sequence's termination."""
    lengths = torch.as_tensor(lengths)
    return torch.arange(max_len)[None, :] < lengths[:, None]
