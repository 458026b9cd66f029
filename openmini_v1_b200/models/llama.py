"""Llama-family decoder (dense or MoE FFN, optional DSA) over a paged KV cache.

Per layer:  h += o_proj(attn(rope(qkv_proj(rmsnorm(h)))))
            h += down(silu(gate(x)) * up(x)),  x = rmsnorm(h)     (or MoE)

This is the standard pre-norm residual. The reference's layer adds the
attention output to the *normed* tensor (openmini-server/src/model/inference/
model.rs:2122-2125, residual = normed + attn); ``ModelConfig.architecture ==
"openmini-quirk"`` reproduces that for oracle comparisons, the default is the
standard form.

Tensor parallelism (Megatron): qkv and gate_up are column-parallel (each rank
owns whole heads / FFN columns), o_proj and down are row-parallel and followed
by a sum over the TP group, which is fused into the next RMSNorm's residual
add. KV heads are sharded with the query heads.

Reference call stack restated: openmini-server/src/model/inference/model.rs
1957-2380 (TransformerLayerWeights::forward_with_cache), 3522-3560 (forward,
compute_logits), 813-960 (MoE).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn

from .. import ops
from ..ops import reference as ref
from ..parallel.state import ParallelState
from .config import ModelConfig

_DTYPES = {"bfloat16": torch.bfloat16, "float32": torch.float32, "float16": torch.float16}


@dataclass
class ForwardBatch:
    """Device-side description of one forward pass over T token rows of S sequences."""
    input_ids: torch.Tensor     # [T] int32
    positions: torch.Tensor     # [T] int32
    slots: torch.Tensor         # [T] int32 cache slot per token (-1 = do not write)
    block_tables: torch.Tensor  # [S, max_blocks] int32
    row_seq: torch.Tensor       # [T] int32 sequence index of each row
    row_ctx: torch.Tensor       # [T] int32 keys visible to each row (position + 1)
    max_ctx: int                # upper bound on row_ctx (fixes the attention split count)
    logits_idx: torch.Tensor    # [S'] rows whose logits are wanted
    # RL replay: per-MoE-layer forced expert ids [T, top_k] (None = route normally)
    forced_routing: dict | None = None
    record_routing: dict | None = None
    # prefill query tiles [n, 4] int32 (row_start, rows, seq, keys of the last row) or None
    prefill_tiles: torch.Tensor | None = None
    # multimodal input: (rows int64 [n], embeddings [n, D]) that replace the token embeddings
    embed_override: tuple | None = None


@dataclass
class KVCache:
    k: list                     # per layer [blocks, Hkv_local, 16, head_dim]
    v: list
    num_blocks: int
    block_size: int = 16
    idx_k: list = field(default_factory=list)  # DSA indexer keys per layer [blocks, 16, indexer_dim]


def _shard(n: int, tp: int, what: str) -> int:
    if n % tp:
        raise ValueError(f"{what}={n} not divisible by tp={tp}")
    return n // tp


class DecoderLM(nn.Module):
    def __init__(self, cfg: ModelConfig, par: ParallelState | None = None, device="cpu", dtype=None,
                 seed: int = 0, init_std: float = 0.02, materialize: bool = True, weight_format: str = "bf16"):
        super().__init__()
        self.cfg = cfg
        self.par = par or ParallelState.single()
        self.device = torch.device(device)
        self.dtype = dtype or _DTYPES[cfg.dtype]
        tp = self.par.tp
        self.hq = _shard(cfg.num_heads, tp, "num_heads")
        self.hkv = _shard(cfg.num_kv_heads, tp, "num_kv_heads") if cfg.num_kv_heads >= tp else 1
        self.hd = cfg.head_dim
        self.ffn = _shard(cfg.intermediate_size, tp, "intermediate_size")
        self.vocab_local = cfg.vocab_size // tp if cfg.vocab_size % tp == 0 else cfg.vocab_size
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.inv_freq = ref.inv_freq(cfg.head_dim, cfg.rope_theta).to(self.device)
        if cfg.mla.enabled:
            if cfg.mla.kv_lora_rank != 512 or cfg.mla.qk_rope_dim != 64:
                raise ValueError("MLA: the latent kernel takes kv_lora_rank 512 and qk_rope_dim 64")
            self.mla_inv_freq = ref.inv_freq(cfg.mla.qk_rope_dim, cfg.rope_theta).to(self.device)
        self.weight_format = weight_format
        self.layers = []
        self._comm = None
        self._sp = None
        self._ep = None
        if materialize:
            self.init_random(seed, init_std)

    # ------------------------------------------------------------------ weights
    def _randn(self, gen, *shape, std=0.02):
        t = torch.empty(*shape, dtype=self.dtype, device=self.device)
        if self.device.type == "cuda":
            t.normal_(0.0, std, generator=gen)
        else:
            t.copy_(torch.randn(*shape, generator=gen, dtype=torch.float32) * std)
        return t

    def init_random(self, seed: int = 0, std: float = 0.02):
        """Random-init N(0, std) weights; each TP rank draws only its own shard.
        With a quantised ``weight_format`` each layer is quantised as soon as it
        is drawn, so the full bf16 model never has to fit in memory."""
        cfg = self.cfg
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed * 1000003 + self.par.tp_rank)
        shared = torch.Generator(device=self.device)  # replicated tensors are equal on every TP rank
        shared.manual_seed(seed * 1000003 + 999983)
        D = cfg.hidden_size
        self.embed = self._randn(shared, cfg.vocab_size, D, std=std)
        self.norm = torch.ones(D, dtype=self.dtype, device=self.device)
        self.lm_head = self.embed if cfg.tie_embeddings else self._randn(gen, self.vocab_local, D, std=std)
        self.layers = []
        for i in range(cfg.num_layers):
            L = {
                "attn_norm": torch.ones(D, dtype=self.dtype, device=self.device),
                "ffn_norm": torch.ones(D, dtype=self.dtype, device=self.device),
            }
            if cfg.mla.enabled:
                from .mla import init_mla
                init_mla(self, L, gen, shared, std)
            else:
                L["qkv"] = self._randn(gen, (self.hq + 2 * self.hkv) * self.hd, D, std=std)
                L["o"] = self._randn(gen, D, self.hq * self.hd, std=std)
            if cfg.moe.is_moe_layer(i):
                E, Fe = cfg.moe.num_experts, cfg.moe.expert_ffn
                L["router"] = self._randn(shared, E + cfg.moe.num_zero_experts, D, std=std)
                L["experts_gate_up"] = [self._randn(gen, 2 * Fe, D, std=std) for _ in range(E)]
                L["experts_down"] = [self._randn(gen, D, Fe, std=std) for _ in range(E)]
                ns = cfg.moe.num_shared_experts
                if ns:  # shared experts as one SwiGLU FFN of width ns * Fe (column-parallel under TP)
                    Fs = _shard(ns * Fe, self.par.tp, "shared expert width")
                    L["shared_gate_up"] = self._randn(gen, 2 * Fs, D, std=std)
                    L["shared_down"] = self._randn(gen, D, Fs, std=std)
            else:
                L["gate_up"] = self._randn(gen, 2 * self.ffn, D, std=std)
                L["down"] = self._randn(gen, D, self.ffn, std=std)
            if cfg.dsa.enabled:
                from .dsa import init_indexer
                L.update(init_indexer(self, shared, std))
            if self.weight_format != "bf16":
                from .quantize import quantize_layer
                quantize_layer(L, self.weight_format)
            self.layers.append(L)

    # ------------------------------------------------------------------ cache
    def kv_bytes_per_block(self) -> int:
        el = torch.finfo(self.dtype).bits // 8
        per = (16 * 576 * el) if self.cfg.mla.enabled else 2 * self.hkv * 16 * self.hd * el
        if self.cfg.dsa.enabled:
            per += 16 * self.cfg.dsa.indexer_dim * el
        return per * self.cfg.num_layers

    def allocate_kv(self, num_blocks: int) -> KVCache:
        if self.cfg.mla.enabled:  # one 576-wide latent row per token; no separate values
            k = [torch.zeros(num_blocks, 16, 576, dtype=self.dtype, device=self.device)
                 for _ in range(self.cfg.num_layers)]
            v = [torch.zeros(num_blocks, 0, dtype=self.dtype, device=self.device) for _ in range(self.cfg.num_layers)]
            return KVCache(k=k, v=v, num_blocks=num_blocks)
        shape = (num_blocks, self.hkv, 16, self.hd)
        k = [torch.zeros(shape, dtype=self.dtype, device=self.device) for _ in range(self.cfg.num_layers)]
        v = [torch.zeros(shape, dtype=self.dtype, device=self.device) for _ in range(self.cfg.num_layers)]
        kv = KVCache(k=k, v=v, num_blocks=num_blocks)
        if self.cfg.dsa.enabled:
            kv.idx_k = [torch.zeros(num_blocks, 16, self.cfg.dsa.indexer_dim, dtype=self.dtype, device=self.device)
                        for _ in range(self.cfg.num_layers)]
        return kv

    # ------------------------------------------------------------------ comm
    def set_comm(self, comm):
        """Tensor-parallel transport with ``all_reduce(t)`` and ``all_gather(t, dim)``."""
        self._comm = comm

    def set_ep(self, ep, ep_rank: int | None = None):
        """Expert parallelism (``parallel.expert.ExpertParallel``): keep only this rank's
        experts in every MoE layer and route their tokens with all-to-all."""
        from ..parallel.expert import shard_experts
        self._ep = ep
        if ep is not None and ep.size > 1:
            r = ep.rank if ep_rank is None else ep_rank
            self.layers = [shard_experts(L, ep.size, r) if "router" in L else L for L in self.layers]

    def set_sp(self, sp):
        """Sequence-parallel transport (``parallel.symm``): token-sharded residual stream with
        fused reduce / RMSNorm / all-gather events replacing the all-reduces."""
        self._sp = sp

    def _use_sp(self, T: int) -> bool:
        return (self._sp is not None and self._sp.fits(T) and not self.cfg.mla.enabled
                and self.cfg.sliding_window <= 0
                and not any("router" in L for L in self.layers))

    def _tp_sum(self, t):
        if self.par.tp > 1:
            self._comm.all_reduce(t)
        return t

    # ------------------------------------------------------------------ forward
    def embed_tokens(self, ids):
        return ops.embedding(ids, self.embed)

    def forward(self, fb: ForwardBatch, kv: KVCache) -> torch.Tensor:
        """Returns final-normed hidden states of rows ``fb.logits_idx``: [S', D]."""
        if self.par.tp > 1 and self._use_sp(fb.input_ids.shape[0]) and fb.embed_override is None:
            return self.forward_sp(fb, kv)
        h = self.embed_tokens(fb.input_ids)  # residual stream [T, D]
        if fb.embed_override is not None:  # image features in place of placeholder tokens
            rows, emb = fb.embed_override
            h.index_copy_(0, rows.to(h.device), emb.to(h.dtype))
        delta = None
        for i, L in enumerate(self.layers):
            h, delta = self.layer_forward(i, L, h, delta, fb, kv)
        x = ops.rmsnorm(h, self.norm, self.cfg.rms_eps, delta=delta)
        return x.index_select(0, fb.logits_idx)

    def forward_sp(self, fb: ForwardBatch, kv: KVCache) -> torch.Tensor:
        """Tensor-parallel forward with the residual stream sharded by token rows.

        Rank r keeps the residual of rows [r Tp/W, (r+1) Tp/W) (Tp = T padded to a
        multiple of W). Every row-parallel GEMM writes its partial into the
        transport's partials region (on the GPU: straight into the owner ranks'
        slots from the GEMM epilogue); one event sums the partials of the owned rows,
        updates the residual, applies the next RMSNorm and gathers the normed rows
        of all ranks, which the next column-parallel GEMM reads whole."""
        sp, cfg = self._sp, self.cfg
        T = fb.input_ids.shape[0]
        Tp = sp.padded(T)
        ids = fb.input_ids
        if Tp > T:
            ids = torch.cat([ids, ids.new_zeros(Tp - T)])
        h = self.embed_tokens(ids[sp.own_slice(Tp)]).contiguous()  # own residual rows
        k = 0
        x = sp.reduce_norm(k, h, self.layers[0]["attn_norm"], cfg.rms_eps, Tp, has_partial=False, wait=False)
        for i, L in enumerate(self.layers):
            qkv = sp.linear_ag(x[:T], L["qkv"])
            ops.rope_kv(qkv, fb.positions, fb.slots, kv.k[i], kv.v[i], self.inv_freq, self.hq, self.hkv, self.hd,
                        cfg.rope_mode)
            if cfg.dsa.enabled:  # the indexer reads the gathered rows the QKV GEMM waited for
                from .dsa import dsa_attention
                attn = dsa_attention(self, i, L, x[:T], qkv, fb, kv)
            elif fb.prefill_tiles is not None and self.hd == 128:
                attn = ops.flash_prefill(qkv, kv.k[i], kv.v[i], fb.block_tables, fb.row_seq, fb.row_ctx,
                                         fb.prefill_tiles, self.hq, self.scale)
            else:
                attn = ops.paged_attention(qkv, kv.k[i], kv.v[i], fb.block_tables, fb.row_seq, fb.row_ctx,
                                           self.hq, self.scale, fb.max_ctx)
            k += 1
            sp.linear_rs(attn.view(T, self.hq * self.hd), L["o"], k, Tp)
            x = sp.reduce_norm(k, h, L["ffn_norm"], cfg.rms_eps, Tp, has_partial=True, wait=False)
            act = ops.silu_mul(sp.linear_ag(x[:T], L["gate_up"]))
            k += 1
            sp.linear_rs(act, L["down"], k, Tp)
            last = i + 1 == len(self.layers)
            w_next = self.norm if last else self.layers[i + 1]["attn_norm"]
            x = sp.reduce_norm(k, h, w_next, cfg.rms_eps, Tp, has_partial=True, wait=last)
        return x[:T].index_select(0, fb.logits_idx)

    def layer_forward(self, i, L, h, delta, fb: ForwardBatch, kv: KVCache):
        cfg = self.cfg
        T = h.shape[0]
        a = ops.rmsnorm(h, L["attn_norm"], cfg.rms_eps, delta=delta)
        if cfg.mla.enabled:
            from .mla import mla_attention
            attn = mla_attention(self, i, L, a, fb, kv)
            return self._after_attention(i, L, a, h, attn, fb)
        qkv = ops.linear(a, L["qkv"])
        ops.rope_kv(qkv, fb.positions, fb.slots, kv.k[i], kv.v[i], self.inv_freq, self.hq, self.hkv, self.hd,
                    cfg.rope_mode)
        if cfg.dsa.enabled:
            from .dsa import dsa_attention
            attn = dsa_attention(self, i, L, a, qkv, fb, kv)
        elif cfg.is_local_layer(i):
            from .window import window_attention
            attn = window_attention(self, qkv, kv.k[i], kv.v[i], fb, cfg.sliding_window, cfg.attention_sinks)
        elif fb.prefill_tiles is not None and self.hd == 128:
            attn = ops.flash_prefill(qkv, kv.k[i], kv.v[i], fb.block_tables, fb.row_seq, fb.row_ctx,
                                     fb.prefill_tiles, self.hq, self.scale)
        else:
            attn = ops.paged_attention(qkv, kv.k[i], kv.v[i], fb.block_tables, fb.row_seq, fb.row_ctx, self.hq,
                                       self.scale, fb.max_ctx)
        attn = attn.view(T, self.hq * self.hd)
        return self._after_attention(i, L, a, h, attn, fb)

    def _after_attention(self, i, L, a, h, attn, fb: ForwardBatch):
        cfg = self.cfg
        if cfg.architecture == "openmini-quirk":
            h = a.clone()
        if self.par.tp == 1:
            ops.linear(attn, L["o"], out=h, resid=h)
            d = None
        else:
            d = self._tp_sum(ops.linear(attn, L["o"]))
        x = ops.rmsnorm(h, L["ffn_norm"], cfg.rms_eps, delta=d)
        if "router" in L:
            from .moe import moe_forward
            y = moe_forward(self, i, L, x, fb)
            if self.par.tp == 1:
                h.add_(y)
                return h, None
            return h, self._tp_sum(y)
        gu = ops.linear(x, L["gate_up"])
        act = ops.silu_mul(gu)
        if self.par.tp == 1:
            ops.linear(act, L["down"], out=h, resid=h)
            return h, None
        return h, self._tp_sum(ops.linear(act, L["down"]))

    def sample(self, x: torch.Tensor, temperature, top_p, top_k, rng, want_mask: bool = False):
        """LM head + sampler -> (tokens int32 [B], logprob fp32 [B], packed keep mask or None).

        Under tensor parallelism with a vocabulary-sharded LM head the rows are sampled
        row-parallel instead of gathering every rank's logits everywhere: one all-to-all
        gives rank r the full-vocabulary logits of rows [r B'/W, (r+1) B'/W) (B' = B
        padded to a multiple of W), each rank samples only those rows (a draw depends on
        the request's seed and step only, so it matches an unsplit run), and one all-gather of
        (token, logprob) pairs returns the result to every rank. Per rank this moves
        1/W of the logits and does 1/W of the sampling work."""
        W = self.par.tp
        if W == 1 or self.vocab_local == self.cfg.vocab_size or want_mask:
            return ops.sample(self.logits(x), temperature, top_p, top_k, rng, want_mask)
        B = x.shape[0]
        Bp = (B + W - 1) // W * W
        per = Bp // W
        lg = ops.linear(x, self.lm_head)  # [B, V / W]
        knobs = [temperature, top_p, top_k, rng]
        if Bp > B:
            lg = torch.cat([lg, lg.new_zeros(Bp - B, lg.shape[1])])
            knobs = [torch.cat([k, k[:1].expand(Bp - B, *k.shape[1:])]) for k in knobs]
        recv = self._comm.all_to_all(lg.view(W, per, -1))  # [src rank, my rows, src vocab shard]
        full = recv.permute(1, 0, 2).reshape(per, -1)
        r = self.par.tp_rank
        rows = slice(r * per, (r + 1) * per)
        tok, lp, _ = ops.sample(full, *(k[rows] for k in knobs), want_mask=False)
        pair = torch.stack([tok, lp.view(torch.int32)], dim=1)  # [per, 2] int32
        allp = self._comm.all_gather(pair, dim=0)  # [Bp, 2]
        return allp[:B, 0].contiguous(), allp[:B, 1].contiguous().view(torch.float32), None

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        lg = ops.linear(x, self.lm_head)
        if self.par.tp > 1 and self.vocab_local != self.cfg.vocab_size:
            lg = self._comm.all_gather(lg, dim=-1)
        return lg
