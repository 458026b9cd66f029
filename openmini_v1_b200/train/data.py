"""Training data: JSONL / plain-text datasets, the SFT prompt template with
prompt-token masking, deterministic shuffling and padded batching.

Reference: openmini-server/src/training/dataloader.rs:17-515 (JSONL records with
"text" or "prompt"/"response" (also "instruction"/"input"/"output"), SFT
template, labels of prompt tokens masked, shuffle per epoch, batches padded to
the longest sample and truncated to max_seq_length).
"""
from __future__ import annotations

import json
import random

import torch

from .loss import IGNORE

SFT_TEMPLATE = "### Instruction:\n{prompt}\n\n### Response:\n"


def read_jsonl(path: str):
    out = []
    with open(path, encoding="utf-8") as f:
        for ln, line in enumerate(f, 1):
            line = line.strip()
            if not line:
                continue
            try:
                out.append(json.loads(line))
            except json.JSONDecodeError as e:
                raise ValueError(f"{path}:{ln}: {e}") from e
    return out


def read_text(path: str, chunk_chars: int = 4096):
    with open(path, encoding="utf-8") as f:
        s = f.read()
    return [{"text": s[i:i + chunk_chars]} for i in range(0, len(s), chunk_chars)]


def _encode(tok, text, bos=True):
    try:
        return tok.encode(text, add_bos=bos)
    except TypeError:
        return tok.encode(text)


def _prompt_response(rec: dict):
    if "prompt" in rec:
        return rec["prompt"], rec.get("response", rec.get("completion", ""))
    if "instruction" in rec:
        p = rec["instruction"] + (("\n" + rec["input"]) if rec.get("input") else "")
        return p, rec.get("output", "")
    return None, None


class TokenizedDataset:
    """Records -> (input_ids, labels) with prompt tokens labelled IGNORE (SFT) or all tokens (CLM)."""

    def __init__(self, records, tokenizer, max_seq_length: int = 2048, template: str = SFT_TEMPLATE,
                 add_eos: bool = True):
        self.samples = []
        eos = getattr(tokenizer, "eos_id", None)
        for rec in records:
            p, r = _prompt_response(rec)
            if p is None:
                ids = tokenizer.encode(rec["text"])
                if add_eos and eos is not None:
                    ids = ids + [eos]
                labels = list(ids)
            else:
                pi = tokenizer.encode(template.format(prompt=p))
                ri = _encode(tokenizer, r, bos=False)
                if add_eos and eos is not None:
                    ri = ri + [eos]
                ids = pi + ri
                labels = [IGNORE] * len(pi) + ri
            ids, labels = ids[:max_seq_length], labels[:max_seq_length]
            if len(ids) >= 2:
                self.samples.append((ids, labels))

    def __len__(self):
        return len(self.samples)


class DataLoader:
    """Shuffled (per epoch, seeded) padded batches; optionally only this rank's share (data parallel)."""

    def __init__(self, dataset: TokenizedDataset, batch_size: int, shuffle: bool = True, seed: int = 0,
                 pad_id: int = 0, rank: int = 0, world: int = 1, drop_last: bool = False):
        self.ds, self.bs, self.shuffle, self.seed = dataset, batch_size, shuffle, seed
        self.pad_id, self.rank, self.world, self.drop_last = pad_id, rank, world, drop_last
        self.epoch = 0

    def set_epoch(self, e: int):
        self.epoch = e

    def __len__(self):
        n = len(self.ds) // self.world
        return n // self.bs if self.drop_last else (n + self.bs - 1) // self.bs

    def __iter__(self):
        idx = list(range(len(self.ds)))
        if self.shuffle:
            random.Random(self.seed * 100003 + self.epoch).shuffle(idx)
        idx = idx[self.rank::self.world][: len(self.ds) // self.world]
        for b in range(0, len(idx), self.bs):
            chunk = idx[b:b + self.bs]
            if self.drop_last and len(chunk) < self.bs:
                break
            yield collate([self.ds.samples[i] for i in chunk], self.pad_id)


def collate(samples, pad_id: int = 0):
    L = max(len(s[0]) for s in samples)
    ids = torch.full((len(samples), L), pad_id, dtype=torch.long)
    labels = torch.full((len(samples), L), IGNORE, dtype=torch.long)
    for i, (a, b) in enumerate(samples):
        ids[i, :len(a)] = torch.tensor(a)
        labels[i, :len(b)] = torch.tensor(b)
    return {"input_ids": ids, "labels": labels}
