"""SafeTensors reader / writer (the public format: u64 little-endian header
length, JSON header {name: {dtype, shape, data_offsets}, "__metadata__": {..}},
then the raw little-endian tensor bytes).

Reference: SafeTensors loading of openmini-server/src/training/safetensors.rs:45-789.
"""
from __future__ import annotations

import json
import mmap
import os
import struct

import numpy as np
import torch

_DT = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool,
}
_NAME = {v: k for k, v in _DT.items()}


def save_file(tensors: dict, path: str, metadata: dict | None = None) -> None:
    header = {}
    off = 0
    blobs = []
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        if t.dtype not in _NAME:
            raise TypeError(f"{name}: dtype {t.dtype} not representable in safetensors")
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _NAME[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * (-len(hb) % 8)  # keep the data section 8-byte aligned
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


class SafeTensorsFile:
    """Memory-mapped reader; ``get(name)`` returns a CPU tensor (copy-free view when aligned)."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        (n,) = struct.unpack("<Q", self._mm[:8])
        if n > len(self._mm) - 8:
            raise ValueError(f"{path}: header length {n} exceeds file size")
        self.header = json.loads(self._mm[8:8 + n].decode())
        self.metadata = self.header.pop("__metadata__", {})
        self._base = 8 + n

    def keys(self):
        return list(self.header.keys())

    def get(self, name: str) -> torch.Tensor:
        e = self.header[name]
        dt = _DT[e["dtype"]]
        a, b = e["data_offsets"]
        buf = np.frombuffer(self._mm, dtype=np.uint8, count=b - a, offset=self._base + a)
        t = torch.from_numpy(buf.copy()) if b > a else torch.empty(0, dtype=torch.uint8)
        return t.view(dt).reshape(e["shape"])

    def close(self):
        self._mm.close()
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def load_file(path: str) -> dict:
    with SafeTensorsFile(path) as f:
        return {k: f.get(k) for k in f.keys()}
