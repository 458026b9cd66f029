"""Tensor-parallel transport selection.

``make_tp_comm`` returns the collective object the decoder uses for its
row-parallel reductions and the vocabulary all-gather of the LM head (NCCL
through torch.distributed). ``attach_tp_transport`` installs the transport a
TP decoder runs with:

* ``"symm"``: the fused kernels over symmetric peer memory -- the o-proj and
  down-proj GEMMs store their output tiles straight into the owner rank's
  partials slot over NVLink (GEMM -> reduce-scatter in one kernel) and the
  reduce / residual / RMSNorm / all-gather step is one kernel
  (:mod:`.symm`, ``csrc/comm/symm.cu``); NCCL still carries the LM-head gather.
* ``"nccl"``: every row-parallel output is all-reduced by NCCL (the baseline
  the fused path is measured against).

Reference: openmini-server/src/distributed/tp.rs:506-625 (column / row
parallel linear with their collectives).
"""
from __future__ import annotations

from .comm import CollectiveOps


def make_tp_comm(par, device):
    return CollectiveOps(par.tp_group)


def attach_tp_transport(model, par, device, kind: str = "symm", max_rows: int = 4096):
    """Give a tensor-parallel ``DecoderLM`` its collectives; returns ``kind``."""
    if par.tp <= 1:
        return None
    model.set_comm(make_tp_comm(par, device))
    if kind in ("symm", "symm_push"):
        from .symm import make_sp
        model.set_sp(make_sp(par, device, max_rows=max_rows, dim=model.cfg.hidden_size, push=kind == "symm_push"))
    elif kind != "nccl":
        raise ValueError(f"unknown TP transport {kind!r}")
    return kind
