"""Reward functions (openmini-server/src/rl/reward.rs:9-280: accuracy,
format, composite) plus the benchmark reward of the GRPO configuration:
the fraction of generated tokens that fall in a seeded subset of ids."""
from __future__ import annotations

import re

import torch


class SubsetFractionReward:
    """r = |{t in completion : t in S}| / |completion|, S = ``size`` ids drawn from a seed."""

    def __init__(self, vocab_size: int, size: int = 1000, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        self.ids = torch.randperm(vocab_size, generator=g)[:size]
        self.member = torch.zeros(vocab_size, dtype=torch.bool)
        self.member[self.ids] = True

    def __call__(self, prompt_ids, completion_ids) -> float:
        if not completion_ids:
            return 0.0
        t = torch.as_tensor(completion_ids, dtype=torch.long)
        return float(self.member[t].float().mean())


class AccuracyReward:
    """1.0 when the normalised answer equals the ground truth."""

    def __init__(self, normalize=lambda s: re.sub(r"\s+", " ", s.strip().lower())):
        self.norm = normalize

    def __call__(self, text: str, ground_truth: str) -> float:
        return 1.0 if self.norm(text) == self.norm(ground_truth) else 0.0


class FormatReward:
    """1.0 when the text matches the required pattern (e.g. <think>...</think><answer>...</answer>)."""

    def __init__(self, pattern: str = r"^<think>.*</think>\s*<answer>.*</answer>$"):
        self.re = re.compile(pattern, re.S)

    def __call__(self, text: str, ground_truth: str | None = None) -> float:
        return 1.0 if self.re.match(text.strip()) else 0.0


class CompositeReward:
    def __init__(self, parts):
        self.parts = parts  # [(weight, fn)]

    def __call__(self, *args) -> float:
        return sum(w * f(*args) for w, f in self.parts)
