"""Operator layer.

CUDA tensors run the hand-written sm_100a kernels of ``openmini_v1_b200._C``
(no library GEMM, no Triton, no fallback: a missing extension raises).
CPU tensors run the fp32 statements in :mod:`.reference`, which double as the
numerics oracle.
"""
from __future__ import annotations

import threading

import torch

from .. import _native
from . import reference as ref

__all__ = [
    "DeviceContext", "ctx", "linear", "rmsnorm", "layernorm", "silu_mul", "gelu", "softmax",
    "embedding", "rope_kv", "kv_write", "paged_attention", "sample", "repetition_penalty",
    "check_status",
]


class DeviceContext:
    """Per-device scratch owned by the op layer: a status word that kernels set
    on a bounded-wait timeout or a bounds violation, and growable fp32
    workspaces for split-K GEMM partials and split-KV attention partials."""

    def __init__(self, device: torch.device):
        self.device = device
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self._ws = {}
        self.frozen = False  # set while capturing a CUDA graph: no reallocation allowed

    def semaphores(self) -> torch.Tensor:
        """Zeroed int32 tile counters of the in-kernel split-K reduction (every kernel that
        uses them leaves them zeroed again)."""
        s = self._ws.get("__sem")
        if s is None:
            if self.frozen:
                raise RuntimeError("semaphores first requested during graph capture")
            s = torch.zeros(1 << 16, dtype=torch.int32, device=self.device)
            self._ws["__sem"] = s
        return s

    def workspace(self, name: str, numel: int) -> torch.Tensor:
        buf = self._ws.get(name)
        if buf is None or buf.numel() < numel:
            if self.frozen:
                raise RuntimeError(f"workspace {name!r} too small during graph capture ({numel})")
            buf = torch.empty(max(numel, 1 << 16), dtype=torch.float32, device=self.device)
            self._ws[name] = buf
        return buf


_ctx_lock = threading.Lock()
_ctxs: dict = {}


def ctx(device) -> DeviceContext:
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    key = str(device)
    c = _ctxs.get(key)
    if c is None:
        with _ctx_lock:
            c = _ctxs.get(key)
            if c is None:
                c = DeviceContext(device)
                _ctxs[key] = c
    return c


def check_status(device=None):
    """Raise if any kernel on ``device`` recorded an error (timeout / bounds)."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    c = ctx(device)
    v = int(c.status.item())
    if v != 0:
        c.status.zero_()
        raise RuntimeError(f"device kernel reported error status {v} on {device}")


# Split-K scratch: sized for the largest decode GEMM partial (splits x M x N fp32).
GEMM_WS_FLOATS = 64 << 20


def linear(x: torch.Tensor, w, out: torch.Tensor | None = None, resid: torch.Tensor | None = None,
           peer: list | None = None):
    """y = x @ w^T (+ resid). ``w`` is a bf16 [N, K] tensor or a quantised weight object.

    ``peer`` (CUDA only) = [partials byte offset, rows per rank, this rank, base pointer of
    every rank]: output row m is stored into rank m // rows_per_rank's symmetric buffer
    (slot of this rank) over NVLink and the kernel publishes the epoch when done; ``out``
    then only supplies the row stride."""
    if not isinstance(w, torch.Tensor):
        if peer is not None:
            return w.linear(x, out=out, resid=resid, peer=peer)
        return w.linear(x, out=out, resid=resid)
    if not x.is_cuda:
        y = ref.linear(x, w, resid)
        if out is not None:
            out.copy_(y.reshape(out.shape))
            return out
        return y
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M, N = x2.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    o2 = out.view(-1, N)
    if M == 0:
        return out
    c = ctx(x.device)
    ws = c.workspace("gemm", GEMM_WS_FLOATS)
    r2 = resid.reshape(-1, N) if resid is not None else None
    if peer is not None:
        _native.C().gemm(x2, w, o2, r2, ws, c.status, peer=peer)
    else:
        _native.C().gemm(x2, w, o2, r2, ws, c.status)
    return out


def rmsnorm(x, w, eps, out=None, delta=None):
    """rmsnorm(x [+= delta]) * w. With ``delta`` the residual x is updated in place."""
    if not x.is_cuda:
        y = ref.rmsnorm(x, w, eps, delta)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty_like(x)
    _native.C().rmsnorm(x, delta, w, out, float(eps))
    return out


def layernorm(x, w, b, eps, out=None):
    if not x.is_cuda:
        return ref.layernorm(x, w, b, eps)
    out = torch.empty_like(x) if out is None else out
    _native.C().layernorm(x.contiguous(), w, b, out, float(eps))
    return out


def silu_mul(gu, out=None):
    if not gu.is_cuda:
        return ref.silu_mul(gu)
    F = gu.shape[-1] // 2
    out = torch.empty(*gu.shape[:-1], F, dtype=gu.dtype, device=gu.device) if out is None else out
    _native.C().silu_mul(gu.contiguous(), out)
    return out


def gelu(x):
    if not x.is_cuda:
        return ref.gelu(x)
    y = torch.empty_like(x)
    _native.C().gelu(x.contiguous(), y)
    return y


def softmax(x, scale=1.0):
    if not x.is_cuda:
        return ref.softmax(x, scale)
    y = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    _native.C().softmax(x.contiguous(), y, float(scale))
    return y


def embedding(ids, table, out=None):
    if not ids.is_cuda:
        return ref.embedding(ids, table)
    out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device) if out is None else out
    _native.C().embedding(ids.to(torch.int32), table, out, ctx(ids.device).status)
    return out


def rope_kv(qkv, positions, slots, k_cache, v_cache, inv_freq, Hq, Hkv, D, mode=0):
    if not qkv.is_cuda:
        return ref.rope_kv(qkv, positions, slots, k_cache, v_cache, inv_freq, Hq, Hkv, D, mode)
    _native.C().rope_kv(qkv, positions, slots, k_cache, v_cache, inv_freq, Hq, Hkv, D, mode,
                        ctx(qkv.device).status)


def kv_write(k, v, slots, k_cache, v_cache):
    if not k.is_cuda:
        return ref.kv_write(k, v, slots, k_cache, v_cache)
    _native.C().kv_write(k, v, slots, k_cache, v_cache)


def mla_decode(q, cache, block_tables, row_seq, row_ctx, max_ctx, scale, out=None):
    """Latent attention (absorbed MLA) of q [rows, H, 576] over the paged latent cache
    [blocks, 16, 576] -> [rows, H, 512] (see ``csrc/attn/mla.cu``)."""
    if not q.is_cuda:
        o = ref.mla_decode(q, cache, block_tables, row_seq, row_ctx, scale)
        if out is not None:
            out.copy_(o)
            return out
        return o
    rows, H = q.shape[0], q.shape[1]
    if out is None:
        out = torch.empty(rows, H, 512, dtype=q.dtype, device=q.device)
    c = ctx(q.device)
    ws = c.workspace("mla", _native.C().mla_workspace(rows, H, int(max_ctx)))
    _native.C().mla_decode(q.contiguous(), cache, block_tables, row_seq, row_ctx, out, ws, int(max_ctx),
                           float(scale), c.status)
    return out


def paged_attention(q, k_cache, v_cache, block_tables, row_seq, row_ctx, Hq, scale, max_ctx, out=None, impl=None):
    """Attention of query rows over the paged cache. ``max_ctx`` bounds the split count.

    On the GPU, head_dim 128 with <= 16 query heads per KV head runs the
    tensor-core kernel ("tc"); other shapes run the CUDA-core kernel ("simt")."""
    rows = row_seq.shape[0]
    D = k_cache.shape[3]
    if not q.is_cuda:
        o = ref.paged_attention(q, k_cache, v_cache, block_tables, row_seq, row_ctx, Hq, scale)
        if out is not None:
            out.copy_(o.reshape(out.shape))
            return out
        return o.reshape(rows, Hq * D)
    if out is None:
        out = torch.empty(rows, Hq * D, dtype=q.dtype, device=q.device)
    c = ctx(q.device)
    need = _native.C().paged_attention_workspace(rows, Hq, D, max_ctx)
    ws = c.workspace("attn", need)
    if impl is None:
        impl = "tc" if D == 128 and Hq // k_cache.shape[1] <= 16 else "simt"
    fn = _native.C().paged_attention_tc if impl == "tc" else _native.C().paged_attention
    fn(q.reshape(rows, -1), k_cache, v_cache, block_tables, row_seq, row_ctx, out.view(rows, -1), ws, Hq,
       int(max_ctx), float(scale), c.status)
    return out


def flash_prefill(q, k_cache, v_cache, block_tables, row_seq, row_ctx, tiles, Hq, scale, out=None, lse=None):
    """Causal prefill attention of query tiles (consecutive rows of one sequence) over the
    paged cache; on the GPU the tcgen05 FlashAttention kernel (head_dim 128). With ``lse``
    (fp32 [T, Hq]) the natural-log sum-exp of every row's scaled scores is written too."""
    T = row_seq.shape[0]
    D = k_cache.shape[3]
    if not q.is_cuda:
        o = ref.paged_attention(q, k_cache, v_cache, block_tables, row_seq, row_ctx, Hq, scale)
        if out is not None:
            out.copy_(o.reshape(out.shape))
            return out
        return o.reshape(T, Hq * D)
    if out is None:
        out = torch.empty(T, Hq * D, dtype=q.dtype, device=q.device)
    c = ctx(q.device)
    _native.C().flash_prefill(q.reshape(T, -1), k_cache, v_cache, block_tables, row_ctx, tiles, out.view(T, -1),
                              Hq, float(scale), c.status, lse=lse)
    return out


def sample(logits, temperature, top_p, top_k, rng, want_mask=False):
    """Returns (tokens int32, logprob fp32, packed keep mask int32 [B, ceil(V/32)] or None).

    Each row's random draw depends only on its request's (seed, offset): the same
    request samples the same token whatever the batch or the tensor-parallel split."""
    B, V = logits.shape
    if not logits.is_cuda:
        t, lp, m = ref.sample(logits, temperature, top_p, top_k, rng)
        return t, lp, (ref.pack_mask(m) if want_mask else None)
    tok = torch.empty(B, dtype=torch.int32, device=logits.device)
    lp = torch.empty(B, dtype=torch.float32, device=logits.device)
    mask = torch.empty(B, (V + 31) // 32, dtype=torch.int32, device=logits.device) if want_mask else None
    _native.C().sample(logits, temperature, top_p, top_k, rng, tok, lp, mask)
    return tok, lp, mask


def repetition_penalty(logits, prev, penalty):
    if not logits.is_cuda:
        return ref.repetition_penalty(logits, prev, penalty)
    _native.C().repetition_penalty(logits, prev.to(torch.int32).contiguous(), penalty)
    return logits
