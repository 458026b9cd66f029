"""GGUF <-> DecoderLM weights.

Tensor names follow the llama.cpp GGUF convention (token_embd, blk.N.attn_q,
...) and also accept the reference loader's names
(openmini-server/src/model/inference/quant_loader.rs:24-312:
model.layers.N.attention.q_proj, model.layers.N.ffn.gate_proj, ...).
Loading shards each tensor for the rank's tensor-parallel slice before it
reaches the device. Q4_0 tensors stay 4-bit (their nibbles and fp16 scales are
re-laid into the tiled device format) when the model's weight format is "q4";
INT8 tensors (I8 + "<name>.scale") stay 8-bit for "int8"; anything else is
dequantised to the model dtype.
"""
from __future__ import annotations

import numpy as np
import torch

from ..gguf import quants
from ..gguf.constants import GGMLType
from ..gguf.reader import GGUFReader
from ..gguf.writer import GGUFWriter
from .config import ModelConfig
from .llama import DecoderLM
from .quantize import Int8Weight, Q4Weight

ALIASES = {
    "token_embd.weight": ["model.embed_tokens.weight", "model.embed_tokens"],
    "output_norm.weight": ["model.norm.weight", "model.norm"],
    "output.weight": ["lm_head.weight", "lm_head"],
    "blk.{i}.attn_norm.weight": ["model.layers.{i}.input_layernorm.weight", "model.layers.{i}.input_layernorm"],
    "blk.{i}.ffn_norm.weight": ["model.layers.{i}.post_attention_layernorm.weight",
                                "model.layers.{i}.post_attention_layernorm"],
    "blk.{i}.attn_q.weight": ["model.layers.{i}.attention.q_proj", "model.layers.{i}.self_attn.q_proj.weight"],
    "blk.{i}.attn_k.weight": ["model.layers.{i}.attention.k_proj", "model.layers.{i}.self_attn.k_proj.weight"],
    "blk.{i}.attn_v.weight": ["model.layers.{i}.attention.v_proj", "model.layers.{i}.self_attn.v_proj.weight"],
    "blk.{i}.attn_output.weight": ["model.layers.{i}.attention.o_proj", "model.layers.{i}.self_attn.o_proj.weight"],
    "blk.{i}.ffn_gate.weight": ["model.layers.{i}.ffn.gate_proj", "model.layers.{i}.mlp.gate_proj.weight"],
    "blk.{i}.ffn_up.weight": ["model.layers.{i}.ffn.up_proj", "model.layers.{i}.mlp.up_proj.weight"],
    "blk.{i}.ffn_down.weight": ["model.layers.{i}.ffn.down_proj", "model.layers.{i}.mlp.down_proj.weight"],
    "blk.{i}.ffn_gate_inp.weight": ["model.layers.{i}.moe.router"],
}


class _Src:
    """Tensor source over a GGUF file with alias resolution."""

    def __init__(self, reader: GGUFReader):
        self.r = reader

    def find(self, name: str, i: int | None = None):
        cands = [name] + ALIASES.get(name, [])
        for c in cands:
            c = c.format(i=i) if i is not None else c
            if c in self.r.tensors:
                return self.r.tensors[c]
        return None

    def get(self, name, i=None):
        t = self.find(name, i)
        if t is None:
            raise KeyError(f"tensor {name.format(i=i) if i is not None else name} not found")
        return t


def _rows(t, lo, hi):
    return t[lo:hi]


def _dense(t, model) -> torch.Tensor:
    """The whole GGUF tensor dequantised on the model's device (GPU kernels for the
    common block formats, host readers otherwise)."""
    from ..gguf.device import dequantize_to_device
    return dequantize_to_device(t.raw, t.type, tuple(t.shape), model.device, model.dtype)


def _load_linear(src: _Src, t, model: DecoderLM, row_slice=None, col_slice=None):
    """Return a device weight for GGUF tensor ``t`` [N, K], sliced for tensor parallelism."""
    fmt = model.weight_format
    N, K = t.shape
    r0, r1 = row_slice or (0, N)
    c0, c1 = col_slice or (0, K)
    if fmt == "q4" and t.type == GGMLType.Q4_0 and c0 % 64 == 0 and (c1 - c0) % 64 == 0:
        q, d = quants.split_q4_0(t.raw, N, K)
        q = np.ascontiguousarray(q[r0:r1, c0 // 2:c1 // 2])
        d = np.ascontiguousarray(d[r0:r1, c0 // 32:c1 // 32])
        qt = torch.from_numpy(q).to(model.device)
        st = torch.from_numpy(d.astype(np.float32)).to(torch.bfloat16).to(model.device)
        return Q4Weight.from_parts(qt, st)
    if fmt == "int8" and t.type == GGMLType.I8:
        scale = src.r.tensors.get(t.name + ".scale")
        q = t.raw.view(np.int8).reshape(N, K)[r0:r1, c0:c1]
        if scale is not None and c0 == 0 and c1 == K:
            s = scale.to_numpy().reshape(-1)[r0:r1]
            from .quantize import tile_i8
            qd = torch.from_numpy(np.ascontiguousarray(q)).to(model.device)
            return Int8Weight(tile_i8(qd), torch.from_numpy(s.astype(np.float32)).to(model.device), qd.shape)
    w = _dense(t, model)[r0:r1, c0:c1].contiguous()
    if fmt == "q4":
        return Q4Weight.from_dense(w)
    if fmt == "int8":
        return Int8Weight.from_dense(w)
    return w


def load_gguf_model(path: str, device="cpu", par=None, weight_format="bf16", dtype=None) -> DecoderLM:
    reader = GGUFReader(path)
    cfg = reader.model_config()
    if dtype is None and str(device).startswith("cpu"):
        cfg.dtype = "float32"
    model = DecoderLM(cfg, par=par, device=device, dtype=dtype, materialize=False, weight_format=weight_format)
    src = _Src(reader)
    tp, r = model.par.tp, model.par.tp_rank
    hd = cfg.head_dim

    def dense(name, i=None, rows=None):
        a = _dense(src.get(name, i), model)
        if rows:
            a = a[rows[0]:rows[1]]
        return a.contiguous()

    model.embed = dense("token_embd.weight")
    model.norm = dense("output_norm.weight")
    if src.find("output.weight") is None:
        model.lm_head = model.embed
    else:
        V = model.vocab_local
        model.lm_head = dense("output.weight", rows=(r * V, (r + 1) * V) if V != cfg.vocab_size else None)
    model.layers = []
    for i in range(cfg.num_layers):
        L = {"attn_norm": dense("blk.{i}.attn_norm.weight", i), "ffn_norm": dense("blk.{i}.ffn_norm.weight", i)}
        if cfg.mla.enabled:
            _load_mla(src, model, L, i)
        else:
            _load_qkv(src, model, L, i)
        if src.find("blk.{i}.ffn_gate_inp.weight", i) is not None:
            _load_moe(src, model, L, i)
            model.layers.append(L)
            continue
        F = model.ffn
        g = src.get("blk.{i}.ffn_gate.weight", i).to_numpy()[r * F:(r + 1) * F]
        u = src.get("blk.{i}.ffn_up.weight", i).to_numpy()[r * F:(r + 1) * F]
        L["gate_up"] = _wrap(model, torch.from_numpy(np.concatenate([g, u])))
        L["down"] = _load_linear(src, src.get("blk.{i}.ffn_down.weight", i), model, col_slice=(r * F, (r + 1) * F))
        model.layers.append(L)
    return model


def _load_qkv(src: _Src, model: DecoderLM, L: dict, i: int):
    cfg, tp, r, hd = model.cfg, model.par.tp, model.par.tp_rank, model.cfg.head_dim
    q_rows = (r * model.hq * hd, (r + 1) * model.hq * hd)
    kv_rows = (r * model.hkv * hd, (r + 1) * model.hkv * hd) if cfg.num_kv_heads >= tp else (0, hd)
    # fused qkv: dequantised concatenation keeps the q|k|v row order the kernels expect
    parts = [src.get("blk.{i}.attn_q.weight", i), src.get("blk.{i}.attn_k.weight", i),
             src.get("blk.{i}.attn_v.weight", i)]
    if model.weight_format == "q4" and all(p.type == GGMLType.Q4_0 for p in parts):
        qs, ds = [], []
        for p, rr in zip(parts, (q_rows, kv_rows, kv_rows)):
            qn, dn = quants.split_q4_0(p.raw, *p.shape)
            qs.append(qn[rr[0]:rr[1]])
            ds.append(dn[rr[0]:rr[1]])
        L["qkv"] = Q4Weight.from_parts(torch.from_numpy(np.concatenate(qs)).to(model.device),
                                       torch.from_numpy(np.concatenate(ds).astype(np.float32))
                                       .to(torch.bfloat16).to(model.device))
    else:
        w = np.concatenate([parts[0].to_numpy()[q_rows[0]:q_rows[1]], parts[1].to_numpy()[kv_rows[0]:kv_rows[1]],
                            parts[2].to_numpy()[kv_rows[0]:kv_rows[1]]])
        L["qkv"] = _wrap(model, torch.from_numpy(w))
    o = src.get("blk.{i}.attn_output.weight", i)
    L["o"] = _load_linear(src, o, model, col_slice=(r * model.hq * hd, (r + 1) * model.hq * hd))


def _load_mla(src: _Src, model: DecoderLM, L: dict, i: int):
    """Latent attention of layer i from DeepSeek-style GGUF tensors:
    attn_q [H (dn + dr), D] or attn_q_a [Rq, D] + attn_q_a_norm [Rq] + attn_q_b [H (dn + dr), Rq];
    attn_kv_a_mqa [512 + 64, D] (latent | shared RoPE key); attn_kv_a_norm [512];
    attn_kv_b [H (dn + dv), 512] (per head: dn key rows then dv value rows), or the split
    attn_k_b / attn_v_b (either orientation; told apart by shape); attn_output [D, H dv].
    Heads are split under TP; the latent projection is replicated.
    Reference: MLAWeights of openmini-server/src/model/inference/model.rs:962-1027."""
    cfg, m, tp, r = model.cfg, model.cfg.mla, model.par.tp, model.par.tp_rank
    H, Hl, dn, dr, dv = cfg.num_heads, model.hq, m.qk_nope_dim, m.qk_rope_dim, m.v_head_dim
    heads = slice(r * Hl, (r + 1) * Hl)
    dev, dt = model.device, model.dtype
    f = lambda name: src.get(name, i).to_numpy()  # noqa: E731
    t = lambda a: torch.from_numpy(np.array(a, dtype=np.float32)).to(dt).to(dev)  # noqa: E731  (own copy)
    qrows = (r * Hl * (dn + dr), (r + 1) * Hl * (dn + dr))
    if src.find("blk.{i}.attn_q_a.weight", i) is not None:
        L["mla_q_a"] = t(f("blk.{i}.attn_q_a.weight"))
        L["mla_q_a_norm"] = t(f("blk.{i}.attn_q_a_norm.weight"))
        L["mla_q_b"] = t(f("blk.{i}.attn_q_b.weight")[qrows[0]:qrows[1]])
    else:
        L["mla_q"] = t(f("blk.{i}.attn_q.weight")[qrows[0]:qrows[1]])
    L["mla_dkv"] = t(f("blk.{i}.attn_kv_a_mqa.weight"))
    L["mla_kv_norm"] = t(f("blk.{i}.attn_kv_a_norm.weight"))
    lat = m.kv_lora_rank
    if src.find("blk.{i}.attn_kv_b.weight", i) is not None:
        kvb = f("blk.{i}.attn_kv_b.weight").reshape(H, dn + dv, lat)
        uk, uv = kvb[:, :dn], kvb[:, dn:]
    else:
        uk = f("blk.{i}.attn_k_b.weight").reshape(H, -1)
        uv = f("blk.{i}.attn_v_b.weight").reshape(H, -1)
        kb, vb = src.get("blk.{i}.attn_k_b.weight", i).shape, src.get("blk.{i}.attn_v_b.weight", i).shape
        uk = uk.reshape(H, dn, lat) if kb[-1] == lat else uk.reshape(H, lat, dn).transpose(0, 2, 1)
        uv = uv.reshape(H, dv, lat) if vb[-1] == lat else uv.reshape(H, lat, dv).transpose(0, 2, 1)
    L["mla_uk"], L["mla_uv"] = t(uk[heads]), t(uv[heads])
    L["o"] = _load_linear(src, src.get("blk.{i}.attn_output.weight", i), model,
                          col_slice=(r * Hl * dv, (r + 1) * Hl * dv))


def _load_moe(src: _Src, model: DecoderLM, L: dict, i: int):
    """MoE FFN of layer i from llama.cpp's stacked expert tensors: ffn_gate_inp [E(+Z), D],
    ffn_{gate,up}_exps [E, Fe, D], ffn_down_exps [E, D, Fe] and the optional shared expert
    ffn_{gate,up}_shexp [Fs, D], ffn_down_shexp [D, Fs] (column / row split under TP).
    Reference: the MoE layer weights of openmini-server/src/model/inference/model.rs:813-960."""
    L["router"] = torch.from_numpy(np.array(src.get("blk.{i}.ffn_gate_inp.weight", i).to_numpy(), np.float32)) \
        .to(model.dtype).to(model.device)
    g = src.get("blk.{i}.ffn_gate_exps.weight", i).to_numpy()
    u = src.get("blk.{i}.ffn_up_exps.weight", i).to_numpy()
    d = src.get("blk.{i}.ffn_down_exps.weight", i).to_numpy()
    L["experts_gate_up"] = [_wrap(model, torch.from_numpy(np.concatenate([g[e], u[e]]))) for e in range(g.shape[0])]
    L["experts_down"] = [_wrap(model, torch.from_numpy(np.array(d[e], np.float32))) for e in range(d.shape[0])]
    if src.find("blk.{i}.ffn_gate_shexp.weight", i) is not None:
        tp, r = model.par.tp, model.par.tp_rank
        sg = src.get("blk.{i}.ffn_gate_shexp.weight", i).to_numpy()
        su = src.get("blk.{i}.ffn_up_shexp.weight", i).to_numpy()
        sd = src.get("blk.{i}.ffn_down_shexp.weight", i).to_numpy()
        Fs = sg.shape[0] // tp
        L["shared_gate_up"] = _wrap(model, torch.from_numpy(np.concatenate([sg[r * Fs:(r + 1) * Fs],
                                                                            su[r * Fs:(r + 1) * Fs]])))
        L["shared_down"] = _wrap(model, torch.from_numpy(np.array(sd[:, r * Fs:(r + 1) * Fs], np.float32)))


def _wrap(model, w: torch.Tensor):
    w = w.to(model.dtype).to(model.device).contiguous()
    if model.weight_format == "q4":
        return Q4Weight.from_dense(w)
    if model.weight_format == "int8":
        return Int8Weight.from_dense(w)
    return w


def save_gguf_model(model: DecoderLM, path: str, quant: str = "f32", tokenizer_tokens=None):
    """Write an unsharded DecoderLM (tp = 1) as GGUF (architecture deepseek2 for latent
    attention, llama otherwise). quant: f32 | f16 | bf16 | q4_0 | q8_0 | i8 | q6_k | q5_0 | q8_k
    | iq4_nl; the latent-attention projections are written in f32."""
    cfg = model.cfg
    if model.par.tp != 1:
        raise ValueError("save an unsharded (tp=1) model")
    arch = "deepseek2" if cfg.mla.enabled else "llama"
    w = GGUFWriter(path, arch)
    a = arch + "."
    for k, v in [("embedding_length", cfg.hidden_size), ("block_count", cfg.num_layers),
                 ("attention.head_count", cfg.num_heads), ("attention.head_count_kv", cfg.num_kv_heads),
                 ("feed_forward_length", cfg.intermediate_size), ("context_length", cfg.max_position),
                 ("rope.freq_base", float(cfg.rope_theta)), ("attention.layer_norm_rms_epsilon", float(cfg.rms_eps)),
                 ("vocab_size", cfg.vocab_size)]:
        w.add_kv(a + k, v)
    if cfg.mla.enabled:
        m = cfg.mla
        for k, v in [("attention.kv_lora_rank", m.kv_lora_rank), ("attention.q_lora_rank", m.q_lora_rank),
                     ("attention.key_length", m.qk_nope_dim + m.qk_rope_dim), ("attention.value_length", m.v_head_dim),
                     ("rope.dimension_count", m.qk_rope_dim)]:
            w.add_kv(a + k, v)
    if cfg.moe.num_experts:
        w.add_kv(a + "expert_count", cfg.moe.num_experts)
        w.add_kv(a + "expert_used_count", cfg.moe.top_k)
        w.add_kv(a + "expert_feed_forward_length", cfg.moe.expert_ffn)
        w.add_kv(a + "expert_shared_count", cfg.moe.num_shared_experts)
        w.add_kv(a + "expert_zero_count", cfg.moe.num_zero_experts)
        w.add_kv(a + "moe_dense_prefix", cfg.moe.ffn_prefix_layers)
    w.add_kv("general.name", cfg.name)
    if tokenizer_tokens:
        w.add_kv("tokenizer.ggml.tokens", list(tokenizer_tokens))
    typ = {"f32": GGMLType.F32, "f16": GGMLType.F16, "bf16": GGMLType.BF16, "q4_0": GGMLType.Q4_0,
           "q8_0": GGMLType.Q8_0, "i8": GGMLType.I8, "q6_k": GGMLType.Q6_K, "q5_0": GGMLType.Q5_0,
           "q8_k": GGMLType.Q8_K, "iq4_nl": GGMLType.IQ4_NL}[quant]

    def npf(t):
        if not isinstance(t, torch.Tensor):
            t = t.dequantize()
        return t.float().cpu().numpy()

    def add_lin(name, arr):
        if typ == GGMLType.I8:
            q, s = quants.quantize_int8_rows(arr)
            w.add_tensor(name, q, GGMLType.I8)
            w.add_tensor(name + ".scale", s, GGMLType.F16)
        else:
            w.add_tensor(name, arr, typ)

    w.add_tensor("token_embd.weight", npf(model.embed))
    w.add_tensor("output_norm.weight", npf(model.norm))
    if not cfg.tie_embeddings:
        w.add_tensor("output.weight", npf(model.lm_head))
    D, hd = cfg.hidden_size, cfg.head_dim
    for i, L in enumerate(model.layers):
        w.add_tensor(f"blk.{i}.attn_norm.weight", npf(L["attn_norm"]))
        w.add_tensor(f"blk.{i}.ffn_norm.weight", npf(L["ffn_norm"]))
        if cfg.mla.enabled:
            if "mla_q_a" in L:
                w.add_tensor(f"blk.{i}.attn_q_a.weight", npf(L["mla_q_a"]))
                w.add_tensor(f"blk.{i}.attn_q_a_norm.weight", npf(L["mla_q_a_norm"]))
                w.add_tensor(f"blk.{i}.attn_q_b.weight", npf(L["mla_q_b"]))
            else:
                w.add_tensor(f"blk.{i}.attn_q.weight", npf(L["mla_q"]))
            w.add_tensor(f"blk.{i}.attn_kv_a_mqa.weight", npf(L["mla_dkv"]))
            w.add_tensor(f"blk.{i}.attn_kv_a_norm.weight", npf(L["mla_kv_norm"]))
            kvb = np.concatenate([npf(L["mla_uk"]), npf(L["mla_uv"])], axis=1)  # [H, dn + dv, 512]
            w.add_tensor(f"blk.{i}.attn_kv_b.weight", kvb.reshape(-1, kvb.shape[-1]))
        else:
            qkv = npf(L["qkv"])
            nq, nk = cfg.num_heads * hd, cfg.num_kv_heads * hd
            add_lin(f"blk.{i}.attn_q.weight", qkv[:nq])
            add_lin(f"blk.{i}.attn_k.weight", qkv[nq:nq + nk])
            add_lin(f"blk.{i}.attn_v.weight", qkv[nq + nk:])
        add_lin(f"blk.{i}.attn_output.weight", npf(L["o"]))
        if "router" in L:
            w.add_tensor(f"blk.{i}.ffn_gate_inp.weight", npf(L["router"]))
            gus = np.stack([npf(t) for t in L["experts_gate_up"]])
            Fe = gus.shape[1] // 2
            add_lin(f"blk.{i}.ffn_gate_exps.weight", gus[:, :Fe])
            add_lin(f"blk.{i}.ffn_up_exps.weight", gus[:, Fe:])
            add_lin(f"blk.{i}.ffn_down_exps.weight", np.stack([npf(t) for t in L["experts_down"]]))
            if "shared_gate_up" in L:
                sgu = npf(L["shared_gate_up"])
                Fs = sgu.shape[0] // 2
                add_lin(f"blk.{i}.ffn_gate_shexp.weight", sgu[:Fs])
                add_lin(f"blk.{i}.ffn_up_shexp.weight", sgu[Fs:])
                add_lin(f"blk.{i}.ffn_down_shexp.weight", npf(L["shared_down"]))
            continue
        gu = npf(L["gate_up"])
        F = cfg.intermediate_size
        add_lin(f"blk.{i}.ffn_gate.weight", gu[:F])
        add_lin(f"blk.{i}.ffn_up.weight", gu[F:])
        add_lin(f"blk.{i}.ffn_down.weight", npf(L["down"]))
    w.write()
