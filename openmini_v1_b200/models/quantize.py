"""Weight-only quantised linear weights (4-bit block-32 and INT8 per output channel).

``Q4Weight``: GGUF Q4_0 semantics (value = (q - 8) * d per 32-block, ggml
nibble order: byte i of a block = element i low nibble, element i + 16 high
nibble). ``Int8Weight``: q int8 [N, K], fp32 scale [N] (fp16-representable),
applied in the GEMM epilogue.

Device format: the packed weight is stored pre-tiled, [ceil(N/128)][K/64][tile],
each 128-row x 64-k tile contiguous (Q4 tiles also carry their bf16 block
scales), so the GEMM streams weights with sequential bulk copies.

``linear`` runs the fused dequant tcgen05 GEMM on the GPU and the fp32 oracle
on the CPU. Reference formats: openmini-server/src/model/inference/quant.rs:56-433
(dequantize), openmini-server/src/kernel/cpu/quantized.rs:9-150 (INT8).
"""
from __future__ import annotations

import torch

from .. import _native, ops
from ..ops import reference as ref


def _pad_rows(t: torch.Tensor, mult: int = 128) -> torch.Tensor:
    n = t.shape[0]
    pad = (-n) % mult
    if pad == 0:
        return t
    return torch.cat([t, torch.zeros(pad, *t.shape[1:], dtype=t.dtype, device=t.device)])


def _ggml_to_tile_order(q: torch.Tensor) -> torch.Tensor:
    """Nibbles in ggml Q4_0 order ([rows, K/2]: byte j of a 32-block = element j low,
    element j + 16 high) -> the device order: per 8 consecutive elements one 32-bit
    word with element 2i in bits [4i, 4i+4) and element 2i+1 in bits [16+4i, 16+4i+4),
    so one mask of the word yields a bf16x2 pair of neighbouring elements."""
    rows, k2 = q.shape
    blk = q.view(rows, k2 // 16, 16)
    e = torch.cat([blk & 15, blk >> 4], dim=2).view(rows, k2 // 4, 8)  # [rows, K/8, 8] elements
    b0 = e[..., 0] | (e[..., 2] << 4)
    b1 = e[..., 4] | (e[..., 6] << 4)
    b2 = e[..., 1] | (e[..., 3] << 4)
    b3 = e[..., 5] | (e[..., 7] << 4)
    return torch.stack([b0, b1, b2, b3], dim=2).view(rows, k2)


def _tile_to_ggml_order(t: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`_ggml_to_tile_order`."""
    rows, k2 = t.shape
    w = t.view(rows, k2 // 4, 4)
    e = torch.stack([w[..., 0] & 15, w[..., 2] & 15, w[..., 0] >> 4, w[..., 2] >> 4,
                     w[..., 1] & 15, w[..., 3] & 15, w[..., 1] >> 4, w[..., 3] >> 4], dim=2)
    e = e.reshape(rows, k2 // 16, 32)
    return (e[..., :16] | (e[..., 16:] << 4)).reshape(rows, k2)


def tile_q4(q: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """ggml-order nibbles [N, K/2] + bf16 scales [N, K/32] -> tiles uint8 [ceil(N/128), K/64, 4608].

    Tile (rt, kb) = 128 rows x 32 bytes of nibbles (K block kb, device nibble order,
    see :func:`_ggml_to_tile_order`) followed by the 2 x 128 bf16 scales of its two
    32-blocks, scale index = block * 128 + row."""
    N, K2 = q.shape
    KB = K2 // 32
    qd = _ggml_to_tile_order(q.contiguous())
    qp = _pad_rows(qd).view(-1, 128, KB, 32).permute(0, 2, 1, 3).contiguous().view(-1, KB, 4096)
    sp = _pad_rows(scales.view(torch.int16)).view(-1, 128, KB, 2).permute(0, 2, 3, 1).contiguous()
    sp = sp.view(torch.uint8).view(-1, KB, 512)
    return torch.cat([qp, sp], dim=2).contiguous()


def untile_q4(tiles: torch.Tensor, N: int):
    """Inverse of :func:`tile_q4`: (ggml-order nibbles uint8 [N, K/2], bf16 scales [N, K/32])."""
    NT, KB, _ = tiles.shape
    q = tiles[:, :, :4096].reshape(NT, KB, 128, 32).permute(0, 2, 1, 3).reshape(NT * 128, KB * 32)[:N]
    s = tiles[:, :, 4096:].contiguous().view(torch.int16).view(NT, KB, 2, 128).permute(0, 3, 1, 2)
    s = s.reshape(NT * 128, KB * 2)[:N].contiguous().view(torch.bfloat16)
    return _tile_to_ggml_order(q.contiguous()), s


def tile_i8(q: torch.Tensor) -> torch.Tensor:
    """int8 [N, K] -> tiles uint8 [ceil(N/128), K/64, 8192] of offset-binary bytes (q + 128)."""
    N, K = q.shape
    KB = K // 64
    ob = q.view(torch.uint8) ^ 0x80
    return _pad_rows(ob).view(-1, 128, KB, 64).permute(0, 2, 1, 3).contiguous().view(-1, KB, 8192)


def untile_i8(tiles: torch.Tensor, N: int) -> torch.Tensor:
    NT, KB, _ = tiles.shape
    ob = tiles.view(NT, KB, 128, 64).permute(0, 2, 1, 3).reshape(NT * 128, KB * 64)[:N]
    return (ob ^ 0x80).contiguous().view(torch.int8)


class Q4Weight:
    """4-bit block-32 weight in the tiled device format (see :func:`tile_q4`)."""
    qtype = 0

    def __init__(self, tiles: torch.Tensor, shape):
        self.tiles = tiles
        self.shape = tuple(shape)

    @property
    def device(self):
        return self.tiles.device

    @staticmethod
    def from_dense(w: torch.Tensor) -> "Q4Weight":
        N, K = w.shape
        if K % 64:
            raise ValueError("Q4 needs K % 64 == 0")
        w = w.to(torch.bfloat16).contiguous()
        if w.is_cuda:
            q = torch.empty(N, K // 2, dtype=torch.uint8, device=w.device)
            s = torch.empty(N, K // 32, dtype=torch.bfloat16, device=w.device)
            _native.C().quantize_q4(w, q, s)
        else:
            q, s = ref.quantize_q4(w)
        return Q4Weight(tile_q4(q, s), (N, K))

    @staticmethod
    def from_parts(q: torch.Tensor, scales_bf16: torch.Tensor) -> "Q4Weight":
        return Q4Weight(tile_q4(q, scales_bf16), (q.shape[0], q.shape[1] * 2))

    def parts(self):
        return untile_q4(self.tiles, self.shape[0])

    def dequantize(self) -> torch.Tensor:
        N, K = self.shape
        q, s = self.parts()
        if q.is_cuda:
            out = torch.empty(N, K, dtype=torch.bfloat16, device=self.device)
            _native.C().dequant_q4(q, s, out)
            return out
        return ref.dequant_q4(q, s)

    def nbytes(self):
        return self.tiles.numel()

    def linear(self, x, out=None, resid=None, peer=None, agwait=None):
        if not x.is_cuda:
            y = ref.linear(x, self.dequantize().to(x.dtype), resid)
            if out is not None:
                out.copy_(y)
                return out
            return y
        return _wq_linear(x, self.tiles, None, 0, self.shape[0], out, resid, peer, agwait)

    def waits_in_kernel(self, M: int) -> bool:
        """Whether a GEMM of M rows runs the decode kernel, which can wait for a
        sequence-parallel gather itself (``agwait``)."""
        return M <= 256 and (self.shape[1] // 64) % 4 == 0


class Int8Weight:
    """INT8 per-output-channel weight: tiles uint8 [ceil(N/128), K/64, 8192] + fp32 scale [N]."""
    qtype = 1

    def __init__(self, tiles: torch.Tensor, scale: torch.Tensor, shape):
        self.tiles = tiles
        self.scale = scale
        self.shape = tuple(shape)

    @property
    def device(self):
        return self.tiles.device

    @staticmethod
    def from_dense(w: torch.Tensor) -> "Int8Weight":
        w = w.to(torch.bfloat16).contiguous()
        N, K = w.shape
        if K % 64:
            raise ValueError("INT8 needs K % 64 == 0")
        if w.is_cuda:
            q = torch.empty(N, K, dtype=torch.int8, device=w.device)
            s = torch.empty(N, dtype=torch.float32, device=w.device)
            _native.C().quantize_int8(w, q, s)
        else:
            q, s = ref.quantize_int8(w)
        return Int8Weight(tile_i8(q), s, (N, K))

    @property
    def qweight(self):
        return untile_i8(self.tiles, self.shape[0])

    def dequantize(self) -> torch.Tensor:
        q = self.qweight
        if q.is_cuda:
            out = torch.empty(self.shape, dtype=torch.bfloat16, device=self.device)
            _native.C().dequant_int8(q, self.scale, out)
            return out
        return ref.dequant_int8(q, self.scale)

    def nbytes(self):
        return self.tiles.numel() + self.scale.numel() * 4

    def waits_in_kernel(self, M: int) -> bool:
        return M <= 256 and (self.shape[1] // 64) % 2 == 0

    def linear(self, x, out=None, resid=None, peer=None, agwait=None):
        if not x.is_cuda:
            y = (x.float() @ self.qweight.float().t()) * self.scale
            if resid is not None:
                y = y + resid.float()
            y = y.to(x.dtype)
            if out is not None:
                out.copy_(y)
                return out
            return y
        return _wq_linear(x, self.tiles, self.scale, 1, self.shape[0], out, resid, peer, agwait)


def _wq_linear(x, tiles, scale, qtype, N, out, resid, peer=None, agwait=None):
    x2 = x.reshape(-1, x.shape[-1])
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    c = ops.ctx(x.device)
    ws = c.workspace("gemm", ops.GEMM_WS_FLOATS)
    r2 = resid.reshape(-1, N) if resid is not None else None
    # decode (M <= 256) runs the stream-K kernel: its per-group counters are ``sem``
    kw = {"sem": c.semaphores()}
    if peer is not None:
        kw["peer"] = peer
    if agwait is not None:
        kw["agwait"] = agwait
    _native.C().gemm_wq(x2, tiles, scale, qtype, out.view(-1, N), r2, ws, c.status, **kw)
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
