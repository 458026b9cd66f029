"""High-performance attention pipeline: one entry point that routes an attention
call to the best strategy for its length and device, with per-strategy statistics.

Strategies:
  "flash"      tcgen05 FlashAttention (``parallel.ring_attention.attend``; on the GPU
               the ``csrc/attn/flash_prefill_tc.cu`` kernel for head_dim 128)
  "streaming"  attention sinks + sliding window for sequences beyond
               ``streaming_threshold`` (the first ``sinks`` keys and the last ``window``)
  "standard"   the fp32 statement (CPU, or head sizes the kernel does not take)

Reference counterpart: openmini-server/src/model/inference/high_performance_pipeline.rs
(HighPerfPipelineConfig presets, select_strategy, HighPerfStats) served by
service/http/inference_handlers.rs (/api/v1/inference/compute).
"""
from __future__ import annotations

import math
import time
from collections import Counter
from dataclasses import dataclass, field

import torch

from . import attention_variants as av


@dataclass
class HighPerfPipelineConfig:
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    num_layers: int = 32
    streaming_threshold: int = 8192
    window: int = 4096
    sinks: int = 4
    enable_flash: bool = True
    enable_streaming: bool = True

    @classmethod
    def for_7b(cls):
        return cls(num_heads=32, num_kv_heads=32, num_layers=32)

    @classmethod
    def for_14b(cls):
        return cls(num_heads=40, num_kv_heads=8, num_layers=40)

    @classmethod
    def for_70b(cls):
        return cls(num_heads=64, num_kv_heads=8, num_layers=80)

    def select_strategy(self, seq_len: int, device: torch.device, head_dim: int) -> str:
        if self.enable_streaming and seq_len > self.streaming_threshold:
            return "streaming"
        if self.enable_flash and (device.type == "cpu" or head_dim == 128):
            return "flash"
        return "standard"


@dataclass
class HighPerfStats:
    calls: int = 0
    total_ms: float = 0.0
    tokens: int = 0
    by_strategy: Counter = field(default_factory=Counter)


def streaming_attention(q, k, v, window: int, sinks: int, scale: float):
    T, S = q.shape[0], k.shape[0]
    t = torch.arange(T, device=q.device)[:, None] + (S - T)
    s = torch.arange(S, device=q.device)[None, :]
    mask = (s <= t) & ((s > t - window) | (s < sinks))
    return av._masked_attention(q, k, v, mask[None], scale)


class HighPerformancePipeline:
    def __init__(self, cfg: HighPerfPipelineConfig | None = None):
        self.cfg = cfg or HighPerfPipelineConfig()
        self.stats = HighPerfStats()
        self.current = None

    def forward(self, q, k, v, causal: bool = True, scale: float | None = None):
        """q [T, H, D], k / v [S, Hkv, D] -> ([T, H, D], strategy)."""
        T, H, D = q.shape
        scale = scale or 1.0 / math.sqrt(D)
        strat = self.cfg.select_strategy(k.shape[0], q.device, D)
        t0 = time.perf_counter()
        if strat == "streaming":
            out = streaming_attention(q, k, v, self.cfg.window, self.cfg.sinks, scale)
        elif strat == "flash" and q.is_cuda and q.shape[0] == k.shape[0]:
            from ..parallel.ring_attention import attend
            out, _ = attend(q.to(torch.bfloat16).contiguous(), k.to(torch.bfloat16).contiguous(),
                            v.to(torch.bfloat16).contiguous(), scale, causal=causal)
        else:
            out = av.full_attention(q, k, v, scale, causal)
        if q.is_cuda:
            torch.cuda.synchronize(q.device)
        self.stats.calls += 1
        self.stats.tokens += T
        self.stats.total_ms += (time.perf_counter() - t0) * 1e3
        self.stats.by_strategy[strat] += 1
        self.current = strat
        return out.float(), strat
