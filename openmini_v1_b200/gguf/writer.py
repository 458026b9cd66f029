"""GGUF v3 writer (used to produce the random-init checkpoints of the benchmark configs)."""
from __future__ import annotations

import struct

import numpy as np

from . import quants
from .constants import (GGUF_MAGIC, GGUF_VERSION, KV_ARRAY, KV_BOOL, KV_FLOAT32, KV_FLOAT64, KV_INT32, KV_INT64,
                        KV_STRING, KV_UINT32, KV_UINT64, GGMLType)


def _s(x: str) -> bytes:
    b = x.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _kv_type(v):
    if isinstance(v, bool):
        return KV_BOOL
    if isinstance(v, int):
        return KV_UINT32 if 0 <= v < 2 ** 32 else (KV_INT64 if v < 0 else KV_UINT64)
    if isinstance(v, float):
        return KV_FLOAT32
    if isinstance(v, str):
        return KV_STRING
    if isinstance(v, (list, tuple)):
        return KV_ARRAY
    raise TypeError(type(v))


def _pack_value(t, v):
    if t == KV_BOOL:
        return struct.pack("<B", 1 if v else 0)
    if t == KV_UINT32:
        return struct.pack("<I", v)
    if t == KV_INT32:
        return struct.pack("<i", v)
    if t == KV_UINT64:
        return struct.pack("<Q", v)
    if t == KV_INT64:
        return struct.pack("<q", v)
    if t == KV_FLOAT32:
        return struct.pack("<f", v)
    if t == KV_FLOAT64:
        return struct.pack("<d", v)
    if t == KV_STRING:
        return _s(v)
    if t == KV_ARRAY:
        et = _kv_type(v[0]) if len(v) else KV_UINT32
        if et == KV_UINT32 and any(isinstance(x, int) and (x < 0 or x >= 2 ** 32) for x in v):
            et = KV_INT64
        if et == KV_FLOAT32 and any(not isinstance(x, float) for x in v):
            raise TypeError("mixed array")
        return struct.pack("<IQ", et, len(v)) + b"".join(_pack_value(et, x) for x in v)
    raise TypeError(t)


class GGUFWriter:
    def __init__(self, path: str, arch: str = "llama", alignment: int = 32):
        self.path = path
        self.alignment = alignment
        self.kv = [("general.architecture", arch), ("general.alignment", alignment)]
        self.tensors = []  # (name, ggml dims, type, bytes)

    def add_kv(self, key: str, value):
        self.kv.append((key, value))

    def add_tensor(self, name: str, arr: np.ndarray, typ: GGMLType = GGMLType.F32):
        """``arr`` is row-major [..., cols]; GGUF dims are stored innermost first."""
        a = np.ascontiguousarray(arr)
        dims = list(reversed(a.shape))
        if typ == GGMLType.F32:
            data = a.astype(np.float32).tobytes()
        elif typ == GGMLType.F16:
            data = a.astype(np.float16).tobytes()
        elif typ == GGMLType.BF16:
            data = (a.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
        elif typ == GGMLType.Q4_0:
            data = quants.quantize_q4_0(a).tobytes()
        elif typ == GGMLType.Q8_0:
            data = quants.quantize_q8_0(a).tobytes()
        elif typ == GGMLType.I8:
            data = a.astype(np.int8).tobytes()
        elif typ in _KQ:
            data = _KQ[typ](a).tobytes()
        else:
            raise NotImplementedError(typ)
        self.tensors.append((name, dims, int(typ), data))

    def add_raw(self, name: str, dims_rowmajor, typ: int, data: bytes):
        self.tensors.append((name, list(reversed(dims_rowmajor)), int(typ), data))

    def write(self):
        head = struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(self.tensors), len(self.kv))
        for k, v in self.kv:
            t = _kv_type(v)
            head += _s(k) + struct.pack("<I", t) + _pack_value(t, v)
        off = 0
        infos = b""
        offsets = []
        for name, dims, typ, data in self.tensors:
            offsets.append(off)
            infos += _s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
            infos += struct.pack("<IQ", typ, off)
            off += (len(data) + self.alignment - 1) // self.alignment * self.alignment
        with open(self.path, "wb") as f:
            f.write(head + infos)
            pos = f.tell()
            pad = (-pos) % self.alignment
            f.write(b"\0" * pad)
            for (name, dims, typ, data), o in zip(self.tensors, offsets):
                f.write(data)
                f.write(b"\0" * ((-len(data)) % self.alignment))


def _kq():
    from . import kquants as k
    return {GGMLType.Q5_0: k.quantize_q5_0, GGMLType.Q5_1: k.quantize_q5_1, GGMLType.Q6_K: k.quantize_q6_k,
            GGMLType.Q8_K: k.quantize_q8_k, GGMLType.IQ4_NL: k.quantize_iq4_nl}


_KQ = _kq()
