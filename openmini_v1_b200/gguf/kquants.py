"""Dequantisers (and simple round-to-nearest quantisers) for the remaining GGUF
block formats and the FP8 / FP4 element codecs, vectorised with numpy.

Block layouts follow the public GGUF specification (all little endian):

  Q5_0   (32 el, 22 B): fp16 d | u32 qh (bit j = 5th bit of element j) | 16 B nibbles
                        element j<16 = low nibble of byte j, element j+16 = high nibble;
                        x = (q - 16) d
  Q5_1   (32 el, 24 B): fp16 d | fp16 m | u32 qh | 16 B nibbles;         x = q d + m
  Q8_1   (32 el, 36 B): fp16 d | fp16 s (= d * sum q, unused here) | 32 int8; x = q d
  Q2_K  (256 el, 84 B): 16 B scales (low nibble scale, high nibble min) | 64 B of 2-bit
                        values | fp16 d | fp16 dmin; x = d sc q - dmin m
  Q3_K (256 el, 110 B): 32 B hmask | 64 B low 2 bits | 12 B of 16 packed 6-bit scales | fp16 d;
                        q = low2 - (hbit ? 0 : 4); x = d (sc - 32) q
  Q5_K (256 el, 176 B): fp16 d | fp16 dmin | 12 B 6-bit scales/mins (as Q4_K) | 32 B qh |
                        128 B nibbles; x = d sc q - dmin m
  Q6_K (256 el, 210 B): 128 B low nibbles | 64 B high 2 bits | 16 int8 scales | fp16 d;
                        x = d sc (q - 32)
  Q8_K (256 el, 292 B): f32 d | 256 int8 | 16 int16 block sums;          x = q d
  IQ4_NL (32 el, 18 B): fp16 d | 16 B nibbles (Q4_0 order) indexing a fixed 16-entry
                        non-uniform codebook; x = d * book[q]
  IQ4_XS (256 el, 136 B): fp16 d | u16 scales_h | 4 B scales_l | 128 B nibbles; eight
                        sub-blocks of 32 with 6-bit scales ls (low 4 bits in scales_l,
                        high 2 in scales_h), x = d (ls - 32) book[q]

Within a K-quant super-block, the 2-bit formats walk two halves of 128 elements;
each half reads 32 bytes and takes four bit planes (shift 0, 2, 4, 6), each plane
covering 32 elements split into two 16-element groups with their own scale.

FP8 E4M3 (OCP "fn" variant: bias 7, no infinities, 0x7F/0xFF NaN) and E5M2 (bias 15,
IEEE-like) go through torch's float8 dtypes; FP4 E2M1 (bias 1, values
{0, .5, 1, 1.5, 2, 3, 4, 6}) is decoded from its 3-bit magnitude.

Reference counterparts: openmini-server/src/model/inference/quant.rs:433-856
(Q5_K, Q6_K, Q2_K, Q3_K, Q8_K, FP8, FP4) and :1246-1330 (IQ4_NL / IQ4_XS). The
reference's IQ4 readers use a layout of their own (130-byte blocks with a
dmin); the layouts here are the ones GGUF files actually contain. The IQ1/IQ2/IQ3
lattice formats are not read: their codebooks are large fixed grids that are
not part of the file.
"""
from __future__ import annotations

import numpy as np
import torch

# IQ4 non-linear codebook (part of the GGUF format definition)
IQ4_BOOK = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=np.float32)


def _blocks(raw, n, per, nbytes):
    return np.asarray(raw, dtype=np.uint8).reshape(-1, nbytes)[: n // per]


def _f16(b, lo):
    return b[:, lo:lo + 2].copy().view(np.float16).astype(np.float32)[:, 0]


def _u32(b, lo):
    return b[:, lo:lo + 4].copy().view(np.uint32)[:, 0]


# ----------------------------------------------------------------------------- 32-element formats

def dequantize_q5_0(raw, n):
    b = _blocks(raw, n, 32, 22)
    d = _f16(b, 0)
    qh = _u32(b, 2)
    qs = b[:, 6:22]
    bits = ((qh[:, None] >> np.arange(32, dtype=np.uint32)) & 1).astype(np.uint8)
    q = np.concatenate([qs & 15, qs >> 4], axis=1) | (bits << 4)
    return ((q.astype(np.float32) - 16.0) * d[:, None]).reshape(-1)


def dequantize_q5_1(raw, n):
    b = _blocks(raw, n, 32, 24)
    d, m = _f16(b, 0), _f16(b, 2)
    qh = _u32(b, 4)
    qs = b[:, 8:24]
    bits = ((qh[:, None] >> np.arange(32, dtype=np.uint32)) & 1).astype(np.uint8)
    q = np.concatenate([qs & 15, qs >> 4], axis=1) | (bits << 4)
    return (q.astype(np.float32) * d[:, None] + m[:, None]).reshape(-1)


def dequantize_q8_1(raw, n):
    b = _blocks(raw, n, 32, 36)
    d = _f16(b, 0)
    q = b[:, 4:36].copy().view(np.int8).astype(np.float32)
    return (q * d[:, None]).reshape(-1)


def dequantize_iq4_nl(raw, n):
    b = _blocks(raw, n, 32, 18)
    d = _f16(b, 0)
    qs = b[:, 2:18]
    q = np.concatenate([qs & 15, qs >> 4], axis=1)
    return (IQ4_BOOK[q] * d[:, None]).reshape(-1)


def _split5(x: np.ndarray, q: np.ndarray):
    """q [B, 32] in 0..31 -> (qh u32 [B], nibble bytes [B, 16])."""
    qh = ((q >> 4).astype(np.uint32) << np.arange(32, dtype=np.uint32)).sum(1).astype(np.uint32)
    lo = q & 15
    return qh, (lo[:, :16] | (lo[:, 16:] << 4)).astype(np.uint8)


def quantize_q5_0(x):
    x = np.asarray(x, np.float32).reshape(-1, 32)
    idx = np.abs(x).argmax(-1)
    mx = x[np.arange(x.shape[0]), idx]
    d = (mx / -16.0).astype(np.float16)
    df = d.astype(np.float32)
    inv = np.where(df != 0, 1.0 / np.where(df != 0, df, 1), 0).astype(np.float32)
    q = np.clip(np.floor(x * inv[:, None] + 16.5), 0, 31).astype(np.uint8)
    qh, qs = _split5(x, q)
    out = np.empty((x.shape[0], 22), np.uint8)
    out[:, :2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:6] = qh.view(np.uint8).reshape(-1, 4)
    out[:, 6:] = qs
    return out.reshape(-1)


def quantize_q5_1(x):
    x = np.asarray(x, np.float32).reshape(-1, 32)
    lo, hi = x.min(-1), x.max(-1)
    d = ((hi - lo) / 31.0).astype(np.float16)
    m = lo.astype(np.float16)
    df, mf = d.astype(np.float32), m.astype(np.float32)
    inv = np.where(df != 0, 1.0 / np.where(df != 0, df, 1), 0).astype(np.float32)
    q = np.clip(np.rint((x - mf[:, None]) * inv[:, None]), 0, 31).astype(np.uint8)
    qh, qs = _split5(x, q)
    out = np.empty((x.shape[0], 24), np.uint8)
    out[:, :2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = m.view(np.uint8).reshape(-1, 2)
    out[:, 4:8] = qh.view(np.uint8).reshape(-1, 4)
    out[:, 8:] = qs
    return out.reshape(-1)


def quantize_iq4_nl(x):
    x = np.asarray(x, np.float32).reshape(-1, 32)
    idx = np.abs(x).argmax(-1)
    mx = x[np.arange(x.shape[0]), idx]
    d = (mx / IQ4_BOOK[0]).astype(np.float16)  # the largest magnitude maps to the book's end -127
    df = d.astype(np.float32)
    inv = np.where(df != 0, 1.0 / np.where(df != 0, df, 1), 0).astype(np.float32)
    q = np.abs((x * inv[:, None])[..., None] - IQ4_BOOK).argmin(-1).astype(np.uint8)
    out = np.empty((x.shape[0], 18), np.uint8)
    out[:, :2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


# ----------------------------------------------------------------------------- K-quants (256 elements)

def _planes2(q64: np.ndarray) -> np.ndarray:
    """64 bytes of 2-bit values -> [B, 256] in element order (two halves x four planes x 32)."""
    B = q64.shape[0]
    out = np.empty((B, 2, 4, 32), np.uint8)
    for h in range(2):
        chunk = q64[:, 32 * h:32 * h + 32]
        for p in range(4):
            out[:, h, p] = (chunk >> (2 * p)) & 3
    return out.reshape(B, 256)


def dequantize_q2_k(raw, n):
    b = _blocks(raw, n, 256, 84)
    sc = b[:, 0:16]
    q = _planes2(b[:, 16:80]).astype(np.float32)
    d, dmin = _f16(b, 80), _f16(b, 82)
    s = (sc & 15).astype(np.float32)  # 16 groups of 16 elements, in element order
    m = (sc >> 4).astype(np.float32)
    x = d[:, None, None] * s[:, :, None] * q.reshape(-1, 16, 16) - dmin[:, None, None] * m[:, :, None]
    return x.reshape(-1)


def _q3k_scales(s12: np.ndarray) -> np.ndarray:
    """12 bytes -> 16 six-bit scales: low 4 bits from bytes 0-7 (low nibbles give scales
    0-7, high nibbles 8-15), high 2 bits from bytes 8-11 (bits 2i..2i+1 of byte 8 + i % 4
    belong to scale i, i // 4 choosing the pair)."""
    lo = np.concatenate([s12[:, 0:8] & 15, s12[:, 0:8] >> 4], axis=1)
    hi = np.empty_like(lo)
    for i in range(16):
        hi[:, i] = (s12[:, 8 + i % 4] >> (2 * (i // 4))) & 3
    return (lo | (hi << 4)).astype(np.int32) - 32


def dequantize_q3_k(raw, n):
    b = _blocks(raw, n, 256, 110)
    hmask = b[:, 0:32]
    low = _planes2(b[:, 32:96]).astype(np.int32)
    sc = _q3k_scales(b[:, 96:108]).astype(np.float32)
    d = _f16(b, 108)
    # high bit of element (half h, plane p, lane l) is bit 4h + p of hmask[l]
    hb = np.empty((b.shape[0], 2, 4, 32), np.int32)
    for h in range(2):
        for p in range(4):
            hb[:, h, p] = (hmask >> (4 * h + p)) & 1
    q = low - 4 * (1 - hb.reshape(-1, 256))
    x = d[:, None, None] * sc[:, :, None] * q.reshape(-1, 16, 16).astype(np.float32)
    return x.reshape(-1)


def _k_scale_min6(sc: np.ndarray):
    """8 (scale, min) pairs of 6 bits from the 12-byte Q4_K / Q5_K array."""
    s = np.empty((sc.shape[0], 8), np.float32)
    m = np.empty_like(s)
    for j in range(8):
        if j < 4:
            s[:, j], m[:, j] = sc[:, j] & 63, sc[:, j + 4] & 63
        else:
            s[:, j] = (sc[:, j + 4] & 15) | ((sc[:, j - 4] >> 6) << 4)
            m[:, j] = (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4)
    return s, m


def dequantize_q5_k(raw, n):
    b = _blocks(raw, n, 256, 176)
    d, dmin = _f16(b, 0), _f16(b, 2)
    s, m = _k_scale_min6(b[:, 4:16])
    qh = b[:, 16:48]
    ql = b[:, 48:176]
    q = np.empty((b.shape[0], 8, 32), np.float32)
    for j in range(8):
        nib = (ql[:, (j // 2) * 32:(j // 2) * 32 + 32] >> (4 * (j % 2))) & 15
        q[:, j] = nib + 16 * ((qh >> j) & 1)
    x = d[:, None, None] * s[:, :, None] * q - dmin[:, None, None] * m[:, :, None]
    return x.reshape(-1)


def dequantize_q6_k(raw, n):
    b = _blocks(raw, n, 256, 210)
    ql = b[:, 0:128]
    qh = b[:, 128:192]
    sc = b[:, 192:208].copy().view(np.int8).astype(np.float32)
    d = _f16(b, 208)
    q = np.empty((b.shape[0], 2, 4, 32), np.int32)
    for h in range(2):
        L = ql[:, 64 * h:64 * h + 64]
        H = qh[:, 32 * h:32 * h + 32]
        q[:, h, 0] = (L[:, 0:32] & 15) | (((H >> 0) & 3) << 4)
        q[:, h, 1] = (L[:, 32:64] & 15) | (((H >> 2) & 3) << 4)
        q[:, h, 2] = (L[:, 0:32] >> 4) | (((H >> 4) & 3) << 4)
        q[:, h, 3] = (L[:, 32:64] >> 4) | (((H >> 6) & 3) << 4)
    q = (q - 32).reshape(-1, 16, 16).astype(np.float32)
    return (d[:, None, None] * sc[:, :, None] * q).reshape(-1)


def quantize_q6_k(x):
    """Round-to-nearest Q6_K: per 16-element group an int8 scale relative to the block's d."""
    x = np.asarray(x, np.float32).reshape(-1, 16, 16)
    B = x.shape[0]
    gmax = np.abs(x).max(-1)                                    # [B, 16]
    gscale = gmax / 31.0                                        # group step so |q| <= 31
    d = (gscale.max(-1) / 127.0).astype(np.float16)
    df = d.astype(np.float32)
    dinv = np.where(df > 0, 1.0 / np.where(df > 0, df, 1), 0)
    sc = np.clip(np.rint(gscale * dinv[:, None]), -128, 127).astype(np.int8)
    step = df[:, None] * sc.astype(np.float32)
    sinv = np.where(step != 0, 1.0 / np.where(step != 0, step, 1), 0)
    q = (np.clip(np.rint(x * sinv[..., None]), -32, 31) + 32).astype(np.uint8).reshape(B, 2, 4, 32)
    ql = np.empty((B, 2, 64), np.uint8)
    qh = np.empty((B, 2, 32), np.uint8)
    for h in range(2):
        ql[:, h, 0:32] = (q[:, h, 0] & 15) | ((q[:, h, 2] & 15) << 4)
        ql[:, h, 32:64] = (q[:, h, 1] & 15) | ((q[:, h, 3] & 15) << 4)
        qh[:, h] = (q[:, h, 0] >> 4) | ((q[:, h, 1] >> 4) << 2) | ((q[:, h, 2] >> 4) << 4) | ((q[:, h, 3] >> 4) << 6)
    out = np.empty((B, 210), np.uint8)
    out[:, 0:128] = ql.reshape(B, 128)
    out[:, 128:192] = qh.reshape(B, 64)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return out.reshape(-1)


def dequantize_q8_k(raw, n):
    b = _blocks(raw, n, 256, 292)
    d = b[:, 0:4].copy().view(np.float32)[:, 0]
    q = b[:, 4:260].copy().view(np.int8).astype(np.float32)
    return (q * d[:, None]).reshape(-1)


def quantize_q8_k(x):
    x = np.asarray(x, np.float32).reshape(-1, 256)
    amax = np.abs(x).max(-1)
    d = (amax / 127.0).astype(np.float32)
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1), 0)
    q = np.clip(np.rint(x * inv[:, None]), -127, 127).astype(np.int8)
    bs = q.reshape(-1, 16, 16).astype(np.int16).sum(-1).astype(np.int16)
    out = np.empty((x.shape[0], 292), np.uint8)
    out[:, 0:4] = d.view(np.uint8).reshape(-1, 4)
    out[:, 4:260] = q.view(np.uint8)
    out[:, 260:292] = bs.view(np.uint8).reshape(-1, 32)
    return out.reshape(-1)


def dequantize_iq4_xs(raw, n):
    b = _blocks(raw, n, 256, 136)
    d = _f16(b, 0)
    sh = b[:, 2:4].copy().view(np.uint16)[:, 0].astype(np.int32)
    sl = b[:, 4:8]
    qs = b[:, 8:136]
    x = np.empty((b.shape[0], 8, 32), np.float32)
    for j in range(8):
        ls = ((sl[:, j // 2] >> (4 * (j % 2))) & 15).astype(np.int32) | (((sh >> (2 * j)) & 3) << 4)
        chunk = qs[:, 16 * j:16 * j + 16]
        q = np.concatenate([chunk & 15, chunk >> 4], axis=1)
        x[:, j] = (d * (ls - 32))[:, None] * IQ4_BOOK[q]
    return x.reshape(-1)


# ----------------------------------------------------------------------------- element codecs

def dequantize_fp8(raw, n, fmt: str = "e4m3"):
    dt = torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2
    t = torch.from_numpy(np.ascontiguousarray(np.asarray(raw, dtype=np.uint8)[:n])).view(dt)
    return t.float().numpy()


def quantize_fp8(x, fmt: str = "e4m3"):
    """Round-to-nearest-even, saturating to the format's largest finite value (448 / 57344)."""
    dt = torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2
    lim = 448.0 if fmt == "e4m3" else 57344.0
    t = torch.from_numpy(np.asarray(x, np.float32).reshape(-1)).clamp(-lim, lim).to(dt)
    return t.view(torch.uint8).numpy()


FP4_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def dequantize_fp4(raw, n):
    """E2M1 pairs, low nibble first."""
    b = np.asarray(raw, dtype=np.uint8)
    nib = np.stack([b & 15, b >> 4], axis=-1).reshape(-1)[:n]
    mag = FP4_VALUES[nib & 7]
    return np.where(nib & 8, -mag, mag).astype(np.float32)


def quantize_fp4(x):
    x = np.asarray(x, np.float32).reshape(-1)
    code = np.abs(np.abs(x)[:, None] - FP4_VALUES).argmin(-1).astype(np.uint8) | ((x < 0).astype(np.uint8) << 3)
    if code.size % 2:
        code = np.concatenate([code, np.zeros(1, np.uint8)])
    return (code[0::2] | (code[1::2] << 4)).astype(np.uint8)
