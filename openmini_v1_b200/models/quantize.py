"""Weight-only quantised linear weights (4-bit block-32 and INT8 per output channel).

``Q4Weight``: GGUF Q4_0 semantics (value = (q - 8) * d per 32-block). Device
layout: qweight uint8 [N, K/2] in the ggml nibble order (byte i of a block =
element i low nibble, element i + 16 high nibble) and scales bf16 transposed to
[K/32, N] so a 128-row tile's scales are one contiguous TMA box.
``Int8Weight``: q int8 [N, K], fp32 scale [N] (fp16-representable), applied in
the GEMM epilogue.

``linear`` runs the fused dequant tcgen05 GEMM on the GPU and the fp32 oracle
on the CPU. Reference formats: openmini-server/src/model/inference/quant.rs:56-433
(dequantize), openmini-server/src/kernel/cpu/quantized.rs:9-150 (INT8).
"""
from __future__ import annotations

import torch

from .. import _native, ops
from ..ops import reference as ref


class Q4Weight:
    qtype = 0

    def __init__(self, qweight: torch.Tensor, scales_t: torch.Tensor):
        self.qweight = qweight          # uint8 [N, K/2]
        self.scales_t = scales_t        # bf16 [K/32, N]
        self.shape = (qweight.shape[0], qweight.shape[1] * 2)

    @property
    def device(self):
        return self.qweight.device

    @staticmethod
    def from_dense(w: torch.Tensor) -> "Q4Weight":
        N, K = w.shape
        if K % 32:
            raise ValueError("Q4 needs K % 32 == 0")
        w = w.to(torch.bfloat16).contiguous()
        if w.is_cuda:
            q = torch.empty(N, K // 2, dtype=torch.uint8, device=w.device)
            s = torch.empty(N, K // 32, dtype=torch.bfloat16, device=w.device)
            _native.C().quantize_q4(w, q, s)
        else:
            q, s = ref.quantize_q4(w)
        return Q4Weight(q, s.t().contiguous())

    def dequantize(self) -> torch.Tensor:
        N, K = self.shape
        s = self.scales_t.t().contiguous()
        if self.qweight.is_cuda:
            out = torch.empty(N, K, dtype=torch.bfloat16, device=self.device)
            _native.C().dequant_q4(self.qweight, s, out)
            return out
        return ref.dequant_q4(self.qweight, s)

    def nbytes(self):
        return self.qweight.numel() + self.scales_t.numel() * 2

    def linear(self, x, out=None, resid=None):
        if not x.is_cuda:
            y = ref.linear(x, self.dequantize().to(x.dtype), resid)
            if out is not None:
                out.copy_(y)
                return out
            return y
        return _wq_linear(x, self.qweight, self.scales_t, 0, self.shape[0], out, resid)


class Int8Weight:
    qtype = 1

    def __init__(self, qweight: torch.Tensor, scale: torch.Tensor):
        self.qweight = qweight          # int8 [N, K]
        self.scale = scale              # fp32 [N]
        self.shape = tuple(qweight.shape)

    @property
    def device(self):
        return self.qweight.device

    @staticmethod
    def from_dense(w: torch.Tensor) -> "Int8Weight":
        w = w.to(torch.bfloat16).contiguous()
        N, K = w.shape
        if w.is_cuda:
            q = torch.empty(N, K, dtype=torch.int8, device=w.device)
            s = torch.empty(N, dtype=torch.float32, device=w.device)
            _native.C().quantize_int8(w, q, s)
        else:
            q, s = ref.quantize_int8(w)
        return Int8Weight(q, s)

    def dequantize(self) -> torch.Tensor:
        if self.qweight.is_cuda:
            out = torch.empty(self.shape, dtype=torch.bfloat16, device=self.device)
            _native.C().dequant_int8(self.qweight, self.scale, out)
            return out
        return ref.dequant_int8(self.qweight, self.scale)

    def nbytes(self):
        return self.qweight.numel() + self.scale.numel() * 4

    def linear(self, x, out=None, resid=None):
        if not x.is_cuda:
            y = (x.float() @ self.qweight.float().t()) * self.scale
            if resid is not None:
                y = y + resid.float()
            y = y.to(x.dtype)
            if out is not None:
                out.copy_(y)
                return out
            return y
        return _wq_linear(x, self.qweight, self.scale, 1, self.shape[0], out, resid)


def _wq_linear(x, q, s, qtype, N, out, resid):
    x2 = x.reshape(-1, x.shape[-1])
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    c = ops.ctx(x.device)
    ws = c.workspace("gemm", ops.GEMM_WS_FLOATS)
    r2 = resid.reshape(-1, N) if resid is not None else None
    _native.C().gemm_wq(x2, q, s, qtype, out.view(-1, N), r2, ws, c.status)
    return out


QUANT = {"q4": Q4Weight, "int8": Int8Weight}
LINEAR_KEYS = ("qkv", "o", "gate_up", "down")


def quantize_layer(L: dict, kind: str):
    cls = QUANT[kind]
    for k in LINEAR_KEYS:
        if k in L and isinstance(L[k], torch.Tensor):
            L[k] = cls.from_dense(L[k])
    for k in ("experts_gate_up", "experts_down"):
        if k in L:
            L[k] = [cls.from_dense(w) if isinstance(w, torch.Tensor) else w for w in L[k]]


def quantize_model(model, kind: str):
    """Replace every decoder-layer projection with its quantised form (embeddings and LM head stay bf16)."""
    for L in model.layers:
        quantize_layer(L, kind)
    if model.device.type == "cuda":
        torch.cuda.empty_cache()
    model.weight_format = kind
