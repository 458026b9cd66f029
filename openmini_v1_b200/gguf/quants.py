"""Block (de)quantisers for the GGUF types the framework reads and writes,
vectorised with numpy. Layouts follow the GGUF specification:

  Q4_0 block (18 B): fp16 d, 16 bytes; byte i = q[i] | q[i+16] << 4; x = (q - 8) d
  Q8_0 block (34 B): fp16 d, 32 int8;  x = q d
  Q4_1 block (20 B): fp16 d, fp16 m, 16 bytes; x = q d + m
  Q4_K super-block (144 B): fp16 d, fp16 dmin, 12 bytes of 6-bit scales/mins,
       128 bytes of nibbles over 8 sub-blocks of 32; x = d*sc*q - dmin*m
"""
from __future__ import annotations

import numpy as np

from .constants import BLOCK_SIZES, GGMLType


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    idx = np.abs(x).argmax(-1)
    mx = x[np.arange(x.shape[0]), idx]
    d = (mx / -8.0).astype(np.float16)
    df = d.astype(np.float32)
    inv = np.where(df != 0, 1.0 / np.where(df != 0, df, 1), 0).astype(np.float32)
    q = np.clip(np.floor(x * inv[:, None] + 8.5), 0, 15).astype(np.uint8)
    packed = q[:, :16] | (q[:, 16:] << 4)
    out = np.empty((x.shape[0], 18), dtype=np.uint8)
    out[:, :2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = packed
    return out.reshape(-1)


def dequantize_q4_0(raw: np.ndarray, n: int) -> np.ndarray:
    b = np.asarray(raw, dtype=np.uint8).reshape(-1, 18)[: n // 32]
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    qs = b[:, 2:]
    lo = (qs & 15).astype(np.float32) - 8
    hi = (qs >> 4).astype(np.float32) - 8
    return (np.concatenate([lo, hi], axis=1) * d).reshape(-1)


def split_q4_0(raw: np.ndarray, rows: int, cols: int):
    """Q4_0 bytes of a [rows, cols] tensor -> (nibbles uint8 [rows, cols/2], fp16 scales [rows, cols/32])."""
    b = np.asarray(raw, dtype=np.uint8).reshape(rows, cols // 32, 18)
    d = b[..., :2].copy().view(np.float16).reshape(rows, cols // 32)
    q = b[..., 2:].reshape(rows, cols // 2)
    return np.ascontiguousarray(q), d


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.abs(x).max(-1)
    d = (amax / 127.0).astype(np.float16)
    df = d.astype(np.float32)
    inv = np.where(df != 0, 1.0 / np.where(df != 0, df, 1), 0)
    q = np.clip(np.rint(x * inv[:, None]), -127, 127).astype(np.int8)
    out = np.empty((x.shape[0], 34), dtype=np.uint8)
    out[:, :2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def dequantize_q8_0(raw, n):
    b = np.asarray(raw, dtype=np.uint8).reshape(-1, 34)[: n // 32]
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].copy().view(np.int8).astype(np.float32)
    return (q * d).reshape(-1)


def dequantize_q4_1(raw, n):
    b = np.asarray(raw, dtype=np.uint8).reshape(-1, 20)[: n // 32]
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    m = b[:, 2:4].copy().view(np.float16).astype(np.float32)
    qs = b[:, 4:]
    q = np.concatenate([(qs & 15), (qs >> 4)], axis=1).astype(np.float32)
    return (q * d + m).reshape(-1)


def _k_scale_min(sc: np.ndarray, j: int):
    """6-bit scale / min of sub-block j from the 12-byte packed array (GGUF K-quant layout)."""
    if j < 4:
        return sc[:, j] & 63, sc[:, j + 4] & 63
    s = (sc[:, j + 4] & 0xF) | ((sc[:, j - 4] >> 6) << 4)
    m = (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4)
    return s, m


def dequantize_q4_k(raw, n):
    b = np.asarray(raw, dtype=np.uint8).reshape(-1, 144)[: n // 256]
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    sc = b[:, 4:16]
    qs = b[:, 16:144]
    out = np.empty((b.shape[0], 256), dtype=np.float32)
    for j in range(8):
        s, m = _k_scale_min(sc, j)
        chunk = qs[:, (j // 2) * 32:(j // 2) * 32 + 32]
        q = (chunk & 15) if j % 2 == 0 else (chunk >> 4)
        out[:, j * 32:(j + 1) * 32] = (d * s)[:, None] * q - (dmin * m)[:, None]
    return out.reshape(-1)


def _extra():
    from . import kquants as k
    return {GGMLType.Q5_0: k.dequantize_q5_0, GGMLType.Q5_1: k.dequantize_q5_1, GGMLType.Q8_1: k.dequantize_q8_1,
            GGMLType.Q2_K: k.dequantize_q2_k, GGMLType.Q3_K: k.dequantize_q3_k, GGMLType.Q5_K: k.dequantize_q5_k,
            GGMLType.Q6_K: k.dequantize_q6_k, GGMLType.Q8_K: k.dequantize_q8_k,
            GGMLType.IQ4_NL: k.dequantize_iq4_nl, GGMLType.IQ4_XS: k.dequantize_iq4_xs}


_EXTRA = _extra()


def dequantize(raw: np.ndarray, typ: int, n: int) -> np.ndarray:
    typ = GGMLType(typ)
    if typ == GGMLType.F32:
        return np.frombuffer(raw.tobytes() if isinstance(raw, np.ndarray) else raw, dtype=np.float32, count=n)
    if typ == GGMLType.F16:
        return np.asarray(raw).view(np.float16)[:n].astype(np.float32)
    if typ == GGMLType.BF16:
        u = np.asarray(raw).view(np.uint16)[:n].astype(np.uint32) << 16
        return u.view(np.float32)
    if typ == GGMLType.Q4_0:
        return dequantize_q4_0(raw, n)
    if typ == GGMLType.Q4_1:
        return dequantize_q4_1(raw, n)
    if typ == GGMLType.Q8_0:
        return dequantize_q8_0(raw, n)
    if typ == GGMLType.Q4_K:
        return dequantize_q4_k(raw, n)
    if typ == GGMLType.I8:
        return np.asarray(raw).view(np.int8)[:n].astype(np.float32)
    if typ in _EXTRA:
        return _EXTRA[typ](raw, n)
    raise NotImplementedError(f"dequantisation of {typ.name} is not implemented")


def nbytes(typ: int, n: int) -> int:
    per, by = BLOCK_SIZES[GGMLType(typ)]
    if n % per:
        raise ValueError(f"{GGMLType(typ).name}: {n} elements not a multiple of block {per}")
    return n // per * by


def quantize_int8_rows(x: np.ndarray):
    """Per-row symmetric INT8: (q int8 [N, K], fp16 scale [N]) with scale = absmax / 127."""
    x = np.asarray(x, dtype=np.float32)
    s = (np.abs(x).max(-1) / 127.0).astype(np.float16)
    sf = s.astype(np.float32)
    inv = np.where(sf > 0, 1.0 / np.where(sf > 0, sf, 1), 0)
    q = np.clip(np.rint(x * inv[:, None]), -127, 127).astype(np.int8)
    return q, s
