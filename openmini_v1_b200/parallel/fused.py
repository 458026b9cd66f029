"""Tensor-parallel transport selection.

``make_tp_comm`` returns the object the decoder uses for its row-parallel
reductions and the vocabulary all-gather of the LM head. The current transport
is NCCL through torch.distributed (NVLS / NVLink 5 selected by NCCL itself);
the fused GEMM + reduce-scatter kernels over symmetric peer memory replace it
per layer when built.
"""
from __future__ import annotations

from .comm import CollectiveOps


def make_tp_comm(par, device):
    return CollectiveOps(par.tp_group)
