"""Python side of the C ABI (include/openmini_b200.h, csrc/runtime/capi.cpp).

A context is one token sequence with its own paged KV cache (blocks laid out
linearly), so ``decode`` / ``sample_token`` / ``get_logits`` give the
step-by-step control of the C API while ``generate`` runs the whole loop.
Everything runs through DecoderLM, the kernels and the device sampler.
"""
from __future__ import annotations

import time

import torch

from . import ops
from .engine.tokenizer import ByteTokenizer
from .models.llama import DecoderLM, ForwardBatch

_models: dict = {}
_ctxs: dict = {}
_next = [1]
_log_cb = [None]


def _id():
    _next[0] += 1
    return _next[0]


def log(level: int, text: str):
    if _log_cb[0] is not None:
        _log_cb[0](level, text)


def set_log(fn):
    _log_cb[0] = fn


def load_model(path: str, n_ctx: int, device_id: int, quant: str) -> int:
    dev = torch.device("cpu") if device_id < 0 or not torch.cuda.is_available() else torch.device("cuda", device_id)
    quant = quant or "bf16"
    if path.startswith("preset:"):
        from .models.config import preset
        cfg = preset(path.split(":", 1)[1])
        m = DecoderLM(cfg, device=dev, weight_format=quant if dev.type == "cuda" else "bf16")
        tok = ByteTokenizer()
    else:
        from .engine.tokenizer import GGUFTokenizer
        from .gguf.reader import GGUFReader
        from .models.loader import load_gguf_model
        m = load_gguf_model(path, device=dev, weight_format=quant if dev.type == "cuda" else "bf16")
        try:
            tok = GGUFTokenizer.from_gguf(GGUFReader(path))
        except Exception:
            tok = ByteTokenizer()
    h = _id()
    _models[h] = {"model": m, "tok": tok, "n_ctx": n_ctx or 4096, "quant": quant}
    log(1, f"loaded {path} on {dev} ({quant})")
    return h


def free_model(h: int):
    _models.pop(h, None)


def model_info(h: int) -> dict:
    mm = _models[h]
    m, c = mm["model"], mm["model"].cfg
    n = sum(t.numel() for t in [m.embed, m.lm_head] if isinstance(t, torch.Tensor))
    D, F, hd = c.hidden_size, c.intermediate_size, c.head_dim
    n += c.num_layers * (D * (c.num_heads + 2 * c.num_kv_heads) * hd + c.num_heads * hd * D + 3 * D * F)
    return {"n_params": int(n), "n_layers": c.num_layers, "n_head": c.num_heads, "n_head_kv": c.num_kv_heads,
            "n_embd": D, "n_vocab": c.vocab_size, "n_ff": F, "type": c.name, "quantization": mm["quant"]}


class _Ctx:
    def __init__(self, mm):
        self.mm = mm
        self.m = mm["model"]
        self.n_ctx = mm["n_ctx"]
        self.kv = self.m.allocate_kv((self.n_ctx + 15) // 16)
        self.reset()
        self.reset_stats()

    def reset(self):
        self.tokens = []
        self.logits = None
        self.rng = torch.tensor([[12345, 0]], dtype=torch.int64, device=self.m.device)

    def reset_stats(self):
        self.st = {"prompt_us": 0, "gen_us": 0, "prompt_tokens": 0, "gen_tokens": 0}

    def decode(self, toks, preprocess_only=False):
        n0 = len(self.tokens)
        T = len(toks)
        if T == 0:
            return
        if n0 + T > self.n_ctx:
            raise OverflowError("context full")
        dev = self.m.device
        i32 = dict(dtype=torch.int32, device=dev)
        pos = torch.arange(n0, n0 + T, **i32)
        nb = (self.n_ctx + 15) // 16
        fb = ForwardBatch(torch.tensor(toks, **i32), pos, pos.clone(), torch.arange(nb, **i32)[None],
                          torch.zeros(T, **i32), pos + 1, n0 + T,
                          torch.tensor([T - 1], device=dev))
        x = self.m(fb, self.kv)
        self.tokens += list(toks)
        if not preprocess_only:
            self.logits = self.m.logits(x).float()[0]

    def sample(self, temperature, top_p, top_k):
        if self.logits is None:
            raise RuntimeError("no logits: decode first")
        dev = self.m.device
        t, _, _ = ops.sample(self.logits[None].to(torch.bfloat16 if dev.type == "cuda" else self.logits.dtype),
                             torch.tensor([temperature], device=dev), torch.tensor([top_p], device=dev),
                             torch.tensor([top_k if top_k > 0 else 0], dtype=torch.int32, device=dev), self.rng)
        self.rng[0, 1] += 1
        return int(t[0])


def new_context(h: int) -> int:
    c = _id()
    _ctxs[c] = _Ctx(_models[h])
    return c


def free_context(c: int):
    _ctxs.pop(c, None)


def reset_context(c: int):
    _ctxs[c].reset()


def decode(c: int, toks, preprocess_only: bool):
    ctx = _ctxs[c]
    t0 = time.perf_counter()
    ctx.decode(list(toks), preprocess_only)
    _sync(ctx)
    ctx.st["prompt_us"] += int((time.perf_counter() - t0) * 1e6)
    ctx.st["prompt_tokens"] += len(toks)


def _sync(ctx):
    if ctx.m.device.type == "cuda":
        torch.cuda.synchronize(ctx.m.device)


def sample_token(c: int, temperature: float, top_p: float, top_k: int) -> int:
    return _ctxs[c].sample(temperature, top_p, top_k)


def get_logits(c: int):
    lg = _ctxs[c].logits
    return None if lg is None else lg.detach().float().cpu().contiguous()


def generate(c: int, prompt: str, max_tokens: int, temperature: float, top_p: float, top_k: int) -> dict:
    ctx = _ctxs[c]
    tok = ctx.mm["tok"]
    ids = tok.encode(prompt)
    t0 = time.perf_counter()
    ctx.decode(ids)
    _sync(ctx)
    t1 = time.perf_counter()
    out = []
    eos = getattr(tok, "eos_id", None)
    for _ in range(max(0, max_tokens)):
        t = ctx.sample(temperature, top_p, top_k)
        out.append(t)
        if t == eos or len(ctx.tokens) >= ctx.n_ctx:
            break
        ctx.decode([t])
    _sync(ctx)
    t2 = time.perf_counter()
    ctx.st["prompt_us"] += int((t1 - t0) * 1e6)
    ctx.st["gen_us"] += int((t2 - t1) * 1e6)
    ctx.st["prompt_tokens"] += len(ids)
    ctx.st["gen_tokens"] += len(out)
    return {"tokens": out, "text": tok.decode(out), "prompt_tokens": len(ids), "prompt_us": (t1 - t0) * 1e6,
            "gen_us": (t2 - t1) * 1e6, "total_us": (t2 - t0) * 1e6}


def stats(c: int) -> dict:
    s = _ctxs[c].st
    tot = s["gen_us"]
    mem = torch.cuda.memory_allocated() / 2 ** 20 if torch.cuda.is_available() else 0.0
    return {"total_prompt_us": s["prompt_us"], "total_gen_us": s["gen_us"],
            "total_tokens": s["prompt_tokens"] + s["gen_tokens"],
            "tokens_per_second": s["gen_tokens"] / (tot / 1e6) if tot else 0.0, "gpu_memory_used_mb": mem,
            "n_prompt_tokens_processed": s["prompt_tokens"], "n_tokens_generated": s["gen_tokens"]}


def reset_stats(c: int):
    _ctxs[c].reset_stats()
