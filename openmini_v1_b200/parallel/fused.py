"""Tensor-parallel transport selection.

``make_tp_comm`` returns the collective object the decoder uses for its
row-parallel reductions and the vocabulary all-gather of the LM head (NCCL
through torch.distributed). ``attach_tp_transport`` installs the transport a
TP decoder runs with:

* ``"symm"`` (default, pull): the row-parallel GEMMs (o-proj, down-proj) write their
  partials locally; one kernel per layer step pulls every peer's partials of its own
  rows over NVLink, adds the residual, applies the next RMSNorm and publishes the
  normed rows, and the next column-parallel weight-only GEMM waits for the gathered
  rows inside the kernel (bounded flag wait) before its first TMA load
  (:mod:`.symm`, ``csrc/comm/symm.cu``); NCCL still carries the LM-head collectives.
* ``"symm_push"``: the row-parallel GEMMs store their output tiles straight into the
  owner rank's partials slot over NVLink and publish the epoch themselves
  (GEMM -> reduce-scatter in one kernel).
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
