"""Differentiable wrappers of the native kernels for training.

``linear(x, w)`` computes x @ w^T with the tcgen05 GEMM on CUDA in forward
and backward (dX = dY @ W, dW = dY^T @ X, each expressed as the kernel's
x @ w^T form on transposed copies); on the CPU it is the fp32 torch statement.
"""
from __future__ import annotations

import torch

from .. import ops


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        return ops.linear(x, w)

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        gy = gy.contiguous().to(x.dtype)
        gx = gw = None
        if ctx.needs_input_grad[0]:
            padn = (-gy.shape[1]) % 8  # the output dim becomes the reduction dim (e.g. a 4-expert router)
            g2 = torch.nn.functional.pad(gy, (0, padn)) if padn else gy
            wt = torch.nn.functional.pad(w.t(), (0, padn)) if padn else w.t()
            gx = ops.linear(g2, wt.contiguous())                          # [M, K] = dY @ W
        if ctx.needs_input_grad[1]:
            pad = (-x.shape[0]) % 8  # the token dim becomes the reduction dim: keep rows 16-byte aligned
            xp = torch.nn.functional.pad(x, (0, 0, 0, pad)) if pad else x
            gp = torch.nn.functional.pad(gy, (0, 0, 0, pad)) if pad else gy
            gw = ops.linear(gp.t().contiguous(), xp.t().contiguous())     # [N, K] = dY^T @ X
        return gx, gw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        return x @ w.t()
    shp = x.shape
    y = _Linear.apply(x.reshape(-1, shp[-1]).contiguous(), w)
    return y.reshape(*shp[:-1], w.shape[0])


def rmsnorm(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)
