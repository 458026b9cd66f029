"""Requests, sampling parameters and per-step outputs.

SamplingParams covers the reference sampler's knobs
(openmini-server/src/model/inference/sampler.rs:45-104: temperature, top_k,
top_p, repetition_penalty, seed) plus generation limits and RL capture flags
(sampled-token log-probs and the top-p kept-set mask for Keep-Sampling-Mask,
openmini-server/src/rl/keep_sampling_mask.rs:10-185).
"""
from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0                 # 0 = disabled
    repetition_penalty: float = 1.0
    max_tokens: int = 16
    min_tokens: int = 0
    stop_token_ids: list = field(default_factory=list)
    ignore_eos: bool = False
    seed: int | None = None
    logprobs: bool = False         # return the sampled token's log-prob
    return_sampling_mask: bool = False  # return the kept set of every step (RL replay)
    return_routing: bool = False   # record MoE router choices for every processed token (Keep Routing)

    def validate(self):
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if not 0 < self.top_p <= 1:
            raise ValueError("top_p must be in (0, 1]")
        if self.top_k < 0:
            raise ValueError("top_k must be >= 0")
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if self.repetition_penalty <= 0:
            raise ValueError("repetition_penalty must be > 0")


class RequestStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"
    ABORTED = "aborted"


_ids = itertools.count()


@dataclass(eq=False)  # identity semantics: requests are compared and hashed by object
class Request:
    request_id: str
    prompt_token_ids: list
    params: SamplingParams
    priority: int = 0              # larger = less important (preempted first)
    arrival: float = field(default_factory=time.monotonic)
    seq_id: int = field(default_factory=lambda: next(_ids))
    status: RequestStatus = RequestStatus.WAITING
    output_token_ids: list = field(default_factory=list)
    output_logprobs: list = field(default_factory=list)
    sampling_masks: list = field(default_factory=list)
    routing: dict = field(default_factory=dict)   # layer -> [int32 [n, k] per processed chunk]
    num_computed: int = 0          # tokens whose KV is in the cache
    first_token_time: float | None = None
    finish_time: float | None = None
    finish_reason: str | None = None
    num_preemptions: int = 0
    rng_offset: int = 0
    # multimodal prompt: (first prompt position, features [n, hidden]) replacing the
    # embeddings of positions [first, first + n)
    image_embeds: tuple | None = None

    @property
    def all_token_ids(self):
        return self.prompt_token_ids + self.output_token_ids

    def token_slice(self, start: int, end: int) -> list:
        """all_token_ids[start:end] without concatenating the whole prompt."""
        P = len(self.prompt_token_ids)
        if start >= P:
            return self.output_token_ids[start - P:end - P]
        if end <= P:
            return self.prompt_token_ids[start:end]
        return self.prompt_token_ids[start:] + self.output_token_ids[:end - P]

    @property
    def num_tokens(self):
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    @property
    def in_prefill(self):
        return self.num_computed < self.num_tokens - (1 if self.output_token_ids else 0)

    @property
    def ttft(self):
        return None if self.first_token_time is None else self.first_token_time - self.arrival

    @property
    def tpot(self):
        n = len(self.output_token_ids)
        if self.finish_time is None or self.first_token_time is None or n < 2:
            return None
        return (self.finish_time - self.first_token_time) / (n - 1)


@dataclass
class RequestOutput:
    request_id: str
    new_token_ids: list
    output_token_ids: list
    finished: bool
    finish_reason: str | None = None
    logprobs: list | None = None
    prompt_tokens: int = 0
