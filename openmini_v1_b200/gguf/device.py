"""GGUF tensors dequantised on the GPU: the packed bytes are uploaded as they are and
expanded to bf16 by ``csrc/quant/gguf_dequant.cu`` (Q4_0, Q8_0, Q4_K, Q5_K, Q6_K);
other types fall back to the host readers."""
from __future__ import annotations

import numpy as np
import torch

from .constants import GGMLType

DEVICE_TYPES = {GGMLType.Q4_0, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q5_K, GGMLType.Q6_K}


def dequantize_to_device(raw, typ: int, shape, device, dtype=torch.bfloat16) -> torch.Tensor:
    """Bytes of a GGUF tensor -> dense tensor of ``shape`` on ``device``."""
    from .. import _native
    from .quants import dequantize
    n = int(np.prod(shape))
    dev = torch.device(device)
    if dev.type == "cuda" and GGMLType(typ) in DEVICE_TYPES:
        r = torch.from_numpy(np.ascontiguousarray(np.asarray(raw, dtype=np.uint8).reshape(-1))).to(dev)
        out = torch.empty(n, dtype=torch.bfloat16, device=dev)
        _native.C().gguf_dequant(r, int(typ), out)
        return out.view(*shape).to(dtype)
    a = np.ascontiguousarray(dequantize(raw, typ, n))
    if not a.flags.writeable:  # an F32 tensor is a view of the read-only file map: own a copy
        a = a.copy()
    return torch.from_numpy(a).view(*shape).to(dtype).to(dev)
