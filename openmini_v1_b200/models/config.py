"""Model architecture configuration and the named presets used by the benchmarks.

Fields mirror what the reference derives from GGUF metadata
(openmini-server/src/model/inference/gguf.rs:2118-2300: embedding_length,
block_count, attention.head_count(_kv), context_length, rope.freq_base,
attention.layer_norm_rms_epsilon) plus the MoE / DSA knobs of
openmini-server/src/config/settings.rs:189-245 and
openmini-server/src/model/inference/dsa.rs:157-166.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field


@dataclass
class MoEConfig:
    num_experts: int = 0           # 0 = dense FFN everywhere
    top_k: int = 2
    expert_ffn: int = 0
    num_shared_experts: int = 0    # always-on SwiGLU experts added to the routed output
    num_zero_experts: int = 0      # zero-computation experts (output = input), LongCat-style
    layer_rule: str = "all"        # "all" | "cyclic" (layer % period == period - 1)
    cycle_period: int = 3
    ffn_prefix_layers: int = 0     # first N layers stay dense
    capacity_factor: float = 1.25

    def is_moe_layer(self, i: int) -> bool:
        if self.num_experts <= 0 or i < self.ffn_prefix_layers:
            return False
        if self.layer_rule == "cyclic":
            return i % self.cycle_period == self.cycle_period - 1
        return True


@dataclass
class DSAConfig:
    enabled: bool = False
    indexer_heads: int = 4
    indexer_dim: int = 64
    top_k: int = 2048
    threshold: int = 1024          # use sparse attention when the context reaches this length


@dataclass
class MLAConfig:
    """Multi-head latent attention: a 512-wide KV latent plus a 64-wide shared RoPE key
    per token (the kernel's fixed widths), per-head no-RoPE query / key width and value
    width; head_dim of the model is ignored for MLA layers."""
    enabled: bool = False
    kv_lora_rank: int = 512
    qk_nope_dim: int = 128
    qk_rope_dim: int = 64
    v_head_dim: int = 128
    q_lora_rank: int = 0       # > 0: q = W_qb RMSNorm(W_qa x) (low-rank query), else q = W_q x


@dataclass
class ModelConfig:
    name: str = "custom"
    vocab_size: int = 32000
    hidden_size: int = 4096
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: int = 32
    head_dim: int = 128
    intermediate_size: int = 11008
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_mode: int = 0             # 0 interleaved pairs (GGUF llama), 1 half split
    max_position: int = 131072
    tie_embeddings: bool = False
    dtype: str = "bfloat16"
    moe: MoEConfig = field(default_factory=MoEConfig)
    dsa: DSAConfig = field(default_factory=DSAConfig)
    mla: MLAConfig = field(default_factory=MLAConfig)
    architecture: str = "llama"
    # sliding-window attention (Gemma-style local layers): 0 = off; with a window,
    # layer i is local unless (i + 1) % sliding_window_global_every == 0 (0: every layer local)
    sliding_window: int = 0
    sliding_window_global_every: int = 0
    # streaming attention (attention sinks): local layers also keep the first N positions
    attention_sinks: int = 0

    def is_local_layer(self, i: int) -> bool:
        if self.sliding_window <= 0:
            return False
        g = self.sliding_window_global_every
        return g <= 0 or (i + 1) % g != 0

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def num_params(self) -> int:
        D, F = self.hidden_size, self.intermediate_size
        attn = D * (self.q_size + 2 * self.kv_size) + self.q_size * D
        n = 0
        for i in range(self.num_layers):
            n += attn + 2 * D
            if self.moe.is_moe_layer(i):
                n += self.moe.num_experts * 3 * D * self.moe.expert_ffn + D * self.moe.num_experts
                n += self.moe.num_shared_experts * 3 * D * self.moe.expert_ffn
            else:
                n += 3 * D * F
        n += self.vocab_size * D * (1 if self.tie_embeddings else 2) + D
        return n

    def to_dict(self):
        return dataclasses.asdict(self)

    @staticmethod
    def from_dict(d):
        d = dict(d)
        moe = MoEConfig(**d.pop("moe", {}))
        dsa = DSAConfig(**d.pop("dsa", {}))
        mla = MLAConfig(**d.pop("mla", {}))
        return ModelConfig(moe=moe, dsa=dsa, mla=mla, **d)


def tiny() -> ModelConfig:
    """Plumbing config: 2 layers, d 256, 4 heads x 64, 2 KV heads, FFN 688, fp32."""
    return ModelConfig(name="tiny-llama", vocab_size=32000, hidden_size=256, num_layers=2, num_heads=4,
                       num_kv_heads=2, head_dim=64, intermediate_size=688, rms_eps=1e-5, rope_theta=10000.0,
                       max_position=4096, dtype="float32")


def llama7b() -> ModelConfig:
    return ModelConfig(name="llama-7b-shape", vocab_size=32000, hidden_size=4096, num_layers=32, num_heads=32,
                       num_kv_heads=32, head_dim=128, intermediate_size=11008, rope_theta=10000.0,
                       max_position=4096)


def dsa14b() -> ModelConfig:
    return ModelConfig(name="14b-dsa-shape", vocab_size=152064, hidden_size=5120, num_layers=40, num_heads=40,
                       num_kv_heads=8, head_dim=128, intermediate_size=13824, rope_theta=1000000.0,
                       max_position=40960, dsa=DSAConfig(enabled=True))


def llama70b() -> ModelConfig:
    return ModelConfig(name="llama-70b-shape", vocab_size=128256, hidden_size=8192, num_layers=80, num_heads=64,
                       num_kv_heads=8, head_dim=128, intermediate_size=28672, rope_theta=500000.0,
                       max_position=8192)


def moe_grpo() -> ModelConfig:
    return ModelConfig(name="moe-grpo-policy", vocab_size=32000, hidden_size=2048, num_layers=24, num_heads=16,
                       num_kv_heads=4, head_dim=128, intermediate_size=1408, rope_theta=10000.0,
                       max_position=4096,
                       moe=MoEConfig(num_experts=16, top_k=2, expert_ffn=1408, layer_rule="all"))


PRESETS = {"tiny": tiny, "llama7b": llama7b, "dsa14b": dsa14b, "llama70b": llama70b, "moe_grpo": moe_grpo}


def preset(name: str) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; choose from {sorted(PRESETS)}")
    return PRESETS[name]()
