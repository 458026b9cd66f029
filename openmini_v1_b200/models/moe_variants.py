"""FFN / MoE variants.

* ``BlockFFN``: the FFN's width is cut into C chunks (each a small SwiGLU expert);
  a router r = RMSNorm(ReLU(W_r x)) scores the chunks per token, chunks with r below
  ``threshold`` are skipped and the rest are scaled by r:
      y = sum_{c : r_c > thr} r_c * W_down_c (SiLU(W_gate_c x) * W_up_c x)
  Tokens are grouped per active chunk, so each chunk runs one GEMM over only the
  tokens that use it (the skipped share is the saved work).
* ``LongCatDualBranch``: a main and an auxiliary FFN branch fused as
  alpha(L) y_main + beta(L) y_aux, with the auxiliary weight growing with the
  sequence length L (sigmoid around ``pivot``); below ``skip_below`` tokens the
  auxiliary branch is a zero-computation expert (not evaluated).

Reference counterparts: openmini-server/src/model/inference/moe/blockffn.rs
(chunk-level sparse FFN with a ReLU + RMSNorm router and a threshold) and
moe/longcat.rs (dual-branch fusion with length-adaptive weights and ZeroExpert
skipping).
"""
from __future__ import annotations

import math

import torch

from .. import ops


def _swiglu(x, gate_up, down):
    return ops.linear(ops.silu_mul(ops.linear(x, gate_up)), down)


class BlockFFN:
    def __init__(self, hidden: int, ffn: int, chunks: int, threshold: float = 0.5, device="cpu",
                 dtype=torch.float32, seed: int = 0, std: float = 0.02):
        if ffn % chunks:
            raise ValueError("ffn must be a multiple of chunks")
        g = torch.Generator().manual_seed(seed)
        r = lambda *s: (torch.randn(*s, generator=g) * std).to(device, dtype)  # noqa: E731
        self.C, self.Fc, self.thr = chunks, ffn // chunks, threshold
        self.router = r(chunks, hidden) * 25
        self.router_norm = torch.ones(chunks, device=device, dtype=dtype)
        self.gate_up = [r(2 * self.Fc, hidden) for _ in range(chunks)]
        self.down = [r(hidden, self.Fc) for _ in range(chunks)]
        self.last_density = 1.0

    def scores(self, x):
        a = torch.relu(ops.linear(x, self.router).float())
        return a * torch.rsqrt(a.pow(2).mean(-1, keepdim=True) + 1e-6) * self.router_norm.float()

    def __call__(self, x):
        r = self.scores(x)
        active = r > self.thr
        self.last_density = float(active.float().mean())
        y = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32, device=x.device)
        for c in range(self.C):
            rows = active[:, c].nonzero().squeeze(1)
            if rows.numel() == 0:
                continue
            yc = _swiglu(x.index_select(0, rows).contiguous(), self.gate_up[c], self.down[c]).float()
            y.index_add_(0, rows, yc * r[rows, c:c + 1])
        return y.to(x.dtype)

    def dense_reference(self, x):
        r = self.scores(x)
        r = torch.where(r > self.thr, r, torch.zeros_like(r))
        y = sum(_swiglu(x, self.gate_up[c], self.down[c]).float() * r[:, c:c + 1] for c in range(self.C))
        return y.to(x.dtype)


class LongCatDualBranch:
    def __init__(self, hidden: int, ffn_main: int, ffn_aux: int, pivot: int = 4096, width: float = 1024.0,
                 skip_below: int = 512, device="cpu", dtype=torch.float32, seed: int = 0, std: float = 0.02):
        g = torch.Generator().manual_seed(seed)
        r = lambda *s: (torch.randn(*s, generator=g) * std).to(device, dtype)  # noqa: E731
        self.main = (r(2 * ffn_main, hidden), r(hidden, ffn_main))
        self.aux = (r(2 * ffn_aux, hidden), r(hidden, ffn_aux))
        self.pivot, self.width, self.skip_below = pivot, width, skip_below
        self.aux_evaluated = 0

    def weights(self, seq_len: int):
        beta = 1.0 / (1.0 + math.exp(-(seq_len - self.pivot) / self.width))
        return 1.0 - 0.5 * beta, 0.5 * beta

    def __call__(self, x, seq_len: int):
        a, b = self.weights(seq_len)
        y = _swiglu(x, *self.main).float() * a
        if seq_len >= self.skip_below:
            self.aux_evaluated += 1
            y = y + _swiglu(x, *self.aux).float() * b
        return y.to(x.dtype)
