"""Dynamic memory network of the serving engine, three levels:

* ``InstantMemory``: the live KV of a session, held by the engine. Saving a session
  writes its tokens and KV (``engine.kv_swap.save_session``); restoring continues it
  without a prefill.
* ``ShortTermMemory``: per session, the most recent conversation turns that fit a
  token budget (oldest turns fall out first).
* ``LongTermMemory``: a vector store of past turns and facts with an HNSW index,
  persisted to one file; ``embed_fn(text) -> vector`` (default: mean of the
  language model's input embeddings of the text's tokens).
* ``MemoryManager``: builds the context of a new prompt from the long-term hits
  above ``min_score`` followed by the short-term window, and records every turn.

Reference counterpart: openmini-server/src/model/inference/memory/{instant,
short_term,long_term,hnsw,persistence,manager}.rs.
"""
from __future__ import annotations

import pickle
import time
from collections import deque
from dataclasses import dataclass, field

import numpy as np

from .hnsw import HNSWIndex


class InstantMemory:
    def __init__(self, engine):
        self.eng = engine
        self.saved: dict = {}

    def save(self, session_id: str, request, path: str):
        """Call while the request is live (its KV is freed when it finishes)."""
        from ..engine.kv_swap import save_session
        save_session(self.eng, request, path)
        self.saved[session_id] = path

    def restore(self, session_id: str, params, extra_tokens=None):
        from ..engine.kv_swap import restore_session
        return restore_session(self.eng, self.saved[session_id], f"{session_id}-r{time.time_ns()}", params,
                               extra_tokens)


@dataclass
class Turn:
    role: str
    text: str
    tokens: int
    t: float = field(default_factory=time.time)


class ShortTermMemory:
    def __init__(self, token_budget: int = 2048, count=lambda s: len(s.split())):
        self.budget, self.count = token_budget, count
        self.sessions: dict[str, deque] = {}

    def add(self, session: str, role: str, text: str):
        d = self.sessions.setdefault(session, deque())
        d.append(Turn(role, text, self.count(text)))
        while sum(t.tokens for t in d) > self.budget and len(d) > 1:
            d.popleft()

    def window(self, session: str) -> list:
        return list(self.sessions.get(session, ()))

    def clear(self, session: str):
        self.sessions.pop(session, None)


class LongTermMemory:
    def __init__(self, embed_fn, dim: int, path: str | None = None, M: int = 16):
        self.embed_fn, self.path = embed_fn, path
        self.index = HNSWIndex(dim, M=M)
        self.items: list[dict] = []
        if path:
            try:
                with open(path, "rb") as f:
                    s = pickle.load(f)
                self.index, self.items = HNSWIndex.from_state(s["index"]), s["items"]
            except FileNotFoundError:
                pass

    def add(self, text: str, meta: dict | None = None) -> int:
        i = self.index.add(self.embed_fn(text))
        self.items.append({"text": text, "meta": meta or {}, "t": time.time()})
        return i

    def search(self, query: str, k: int = 5):
        return [(s, self.items[i]) for s, i in self.index.search(self.embed_fn(query), k)]

    def save(self):
        if self.path:
            with open(self.path, "wb") as f:
                pickle.dump({"index": self.index.state(), "items": self.items}, f)


def model_embed_fn(model, tokenizer):
    """Mean of the model's input embeddings over the text's tokens (a cheap sentence vector)."""
    table = model.embed.float().cpu().numpy()

    def fn(text: str):
        ids = [i for i in tokenizer.encode(text, add_bos=False) if i < table.shape[0]] or [0]
        return table[ids].mean(0)
    return fn


class MemoryManager:
    def __init__(self, short: ShortTermMemory, long: LongTermMemory | None = None, k: int = 3,
                 min_score: float = 0.3):
        self.short, self.long, self.k, self.min_score = short, long, k, min_score

    def record(self, session: str, role: str, text: str, remember: bool = True):
        self.short.add(session, role, text)
        if remember and self.long is not None and role == "user":
            self.long.add(text, {"session": session})

    def context(self, session: str, query: str) -> list:
        """[(role, text)]: recalled long-term items then the recent window."""
        out = []
        if self.long is not None and len(self.long.index):
            recent = {t.text for t in self.short.window(session)}
            for s, item in self.long.search(query, self.k):
                if s >= self.min_score and item["text"] not in recent:
                    out.append(("memory", item["text"]))
        return out + [(t.role, t.text) for t in self.short.window(session)]
