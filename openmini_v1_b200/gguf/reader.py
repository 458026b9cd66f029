"""GGUF reader: the C++ runtime parses the header / metadata / tensor directory,
numpy memory-maps the data section (no copy until a tensor is requested).

Mirrors GgufFile::{open, get_tensor_data_by_ref, get_model_config}
(openmini-server/src/model/inference/gguf.rs:1357,2062,2118), including the
architecture-prefixed metadata keys and the prefix fallback for unknown
architecture names.
"""
from __future__ import annotations

import numpy as np

from .. import _native
from . import quants
from .constants import GGMLType

# architecture names the loader treats as Llama-style decoders
LLAMA_LIKE = ("llama", "qwen2", "qwen3", "minicpm", "mistral", "mixtral", "yi", "baichuan", "gemma", "phi3",
              "deepseek", "deepseek2", "internlm2", "stablelm", "openmini")


class GGUFTensor:
    def __init__(self, reader, name, dims, typ, offset):
        self.reader = reader
        self.name = name
        self.shape = tuple(reversed(dims))  # row-major
        self.type = GGMLType(typ)
        self.offset = offset
        self.n = int(np.prod(self.shape)) if self.shape else 1

    @property
    def raw(self) -> np.ndarray:
        nb = quants.nbytes(self.type, self.n)
        start = self.reader.data_offset + self.offset
        return self.reader.mm[start:start + nb]

    def to_numpy(self) -> np.ndarray:
        """Dequantised float32 array in row-major shape."""
        return quants.dequantize(self.raw, self.type, self.n).reshape(self.shape)


class GGUFReader:
    def __init__(self, path: str):
        self.path = path
        info = _native.rt().parse_gguf(path)
        self.version = info["version"]
        self.metadata = info["metadata"]
        self.data_offset = info["data_offset"]
        self.mm = np.memmap(path, dtype=np.uint8, mode="r")
        self.tensors = {n: GGUFTensor(self, n, d, t, o) for (n, d, t, o) in info["tensors"]}

    @property
    def architecture(self) -> str:
        return str(self.metadata.get("general.architecture", "llama"))

    def get(self, key, default=None):
        arch = self.architecture
        for k in (f"{arch}.{key}", key):
            if k in self.metadata:
                return self.metadata[k]
        # prefix fallback: any "<something>.<key>"
        for k, v in self.metadata.items():
            if k.endswith("." + key):
                return v
        return default

    def model_config(self):
        from ..models.config import DSAConfig, MLAConfig, ModelConfig, MoEConfig
        D = int(self.get("embedding_length"))
        H = int(self.get("attention.head_count"))
        Hkv = int(self.get("attention.head_count_kv", H))
        hd = int(self.get("attention.key_length", D // H))
        vocab = self.get("vocab_size")
        if vocab is None:
            toks = self.metadata.get("tokenizer.ggml.tokens")
            vocab = len(toks) if toks else self.tensors["token_embd.weight"].shape[0]
        moe = MoEConfig()
        E = self.get("expert_count")
        if E:
            moe = MoEConfig(num_experts=int(E), top_k=int(self.get("expert_used_count", 2)),
                            expert_ffn=int(self.get("expert_feed_forward_length", self.get("feed_forward_length"))),
                            num_shared_experts=int(self.get("expert_shared_count", 0)),
                            num_zero_experts=int(self.get("expert_zero_count", 0)),
                            ffn_prefix_layers=int(self.get("moe_dense_prefix", 0)))
        dsa = DSAConfig(enabled=bool(self.get("dsa.enabled", False)))
        if dsa.enabled:
            dsa.indexer_heads = int(self.get("dsa.indexer_heads", 4))
            dsa.indexer_dim = int(self.get("dsa.indexer_dim", 64))
            dsa.top_k = int(self.get("dsa.top_k", 2048))
        mla = MLAConfig()
        if self.get("attention.kv_lora_rank"):  # DeepSeek-style latent attention (deepseek2 keys)
            dr = int(self.get("rope.dimension_count", 64))
            mla = MLAConfig(enabled=True, kv_lora_rank=int(self.get("attention.kv_lora_rank")), qk_rope_dim=dr,
                            qk_nope_dim=hd - dr, v_head_dim=int(self.get("attention.value_length", hd - dr)),
                            q_lora_rank=int(self.get("attention.q_lora_rank", 0) or 0))
        return ModelConfig(
            name=str(self.metadata.get("general.name", self.architecture)), vocab_size=int(vocab), hidden_size=D,
            num_layers=int(self.get("block_count")), num_heads=H, num_kv_heads=Hkv, head_dim=hd,
            intermediate_size=int(self.get("feed_forward_length", 4 * D)),
            rms_eps=float(self.get("attention.layer_norm_rms_epsilon", 1e-5)),
            rope_theta=float(self.get("rope.freq_base", 10000.0)),
            max_position=int(self.get("context_length", 4096)),
            tie_embeddings="output.weight" not in self.tensors, moe=moe, dsa=dsa, mla=mla)
