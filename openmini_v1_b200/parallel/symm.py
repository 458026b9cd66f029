"""Sequence-parallel transport of the tensor-parallel decoder over symmetric
peer memory.

Under tensor parallelism the decoder's residual stream is sharded by token
rows: with W ranks and T rows (padded to a multiple of W), rank r owns rows
[r T/W, (r+1) T/W). Each row-parallel GEMM (o-proj, down-proj) writes its
partial output into this rank's *partials* region; one event then

  1. publishes "partials written" to every peer (``sp_signal``),
  2. for every owned row sums the W partial rows read from the peers over
     NVLink, adds them to the residual row, applies RMSNorm and stores the
     normed row into every rank's *gather* region (``sp_reduce_norm_gather``),
  3. waits until every rank's normed rows have arrived (``sp_wait``),

after which the next column-parallel GEMM (QKV, gate-up, LM head) reads the full
normed activations locally.

With ``push=True`` (the default) step 1 and the NVLink half of step 2 move into
the row-parallel GEMM (``linear_rs``): its epilogue stores every output tile
into the owner rank's partials slot over NVLink as the tile leaves TMEM and its
last CTA publishes the epoch, so GEMM and reduce-scatter are one kernel whose
transfer overlaps the remaining tiles' math; the reduce then sums W local
slots. Reduce-scatter, residual add, RMSNorm and
all-gather are one kernel; every byte crosses NVLink once. Regions are
double-buffered by event parity; the flag protocol (every event waits for every
rank's signal of the same event) keeps a fast rank from overwriting a region a
peer still reads.

``SymmetricSP`` runs that protocol with the CUDA kernels of csrc/comm/symm.cu
on peer-mapped buffers (CUDA IPC). ``EmulatedSP`` runs the same interface with
torch.distributed collectives (gloo on CPU), so the sharded-residual model code
is testable without GPUs.

Reference counterpart: TensorParallelManager's row split -> all_reduce and
column split -> all_gather (openmini-server/src/distributed/tp.rs:506-625).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _native
from ..ops import reference as ref

_CTRL = 256


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class _SPBase:
    world: int
    rank: int
    max_rows: int
    dim: int

    def padded(self, T: int) -> int:
        return (T + self.world - 1) // self.world * self.world

    def fits(self, T: int) -> bool:
        return self.padded(T) <= self.max_rows

    def own_slice(self, Tp: int) -> slice:
        n = Tp // self.world
        return slice(self.rank * n, (self.rank + 1) * n)


class SymmetricSP(_SPBase):
    """Peer-mapped buffers + fused reduce / RMSNorm / all-gather kernels (one process per GPU)."""

    def __init__(self, group, device, max_rows: int, dim: int, push: bool = False):
        self.push = push
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("symmetric SP transport supports at most 8 ranks (one NVSwitch domain)")
        self.device = torch.device(device)
        self.max_rows = max_rows
        self.dim = dim
        self.region = _align(max_rows * dim * 2)
        self.nbytes = _CTRL + 4 * self.region
        C = _native.C()
        with torch.cuda.device(self.device):
            self.ptr = C.symm_alloc(self.nbytes)
            h = bytes(C.symm_handle(self.ptr).numpy().tobytes())
            handles = [None] * self.world
            dist.all_gather_object(handles, h, group=group)
            self.bases = []
            self._opened = []
            for r, hb in enumerate(handles):
                if r == self.rank:
                    self.bases.append(self.ptr)
                else:
                    p = C.symm_open(torch.frombuffer(bytearray(hb), dtype=torch.uint8))
                    self.bases.append(p)
                    self._opened.append(p)
        self.status = None

    def _off(self, kind: str, k: int) -> int:
        i = (0 if kind == "p" else 2) + (k & 1)
        return _CTRL + i * self.region

    def partial(self, k: int, rows: int) -> torch.Tensor:
        """This rank's partials region of event ``k`` as a [rows, dim] bf16 tensor."""
        return _native.C().symm_view(self.ptr, self._off("p", k), [rows, self.dim], 0)

    def gathered(self, k: int, rows: int) -> torch.Tensor:
        return _native.C().symm_view(self.ptr, self._off("x", k), [rows, self.dim], 0)

    def linear_rs(self, x: torch.Tensor, w, k: int, Tp: int):
        """Row-parallel GEMM of event ``k`` whose output rows land in their owners' partials
        slots (push mode: fused GEMM -> reduce-scatter; otherwise a local partial)."""
        from .. import ops
        T = x.shape[0]
        out = self.partial(k, Tp)[:T]
        if not self.push:
            return ops.linear(x, w, out=out)
        peer = [self._off("p", k), Tp // self.world, self.rank, *self.bases]
        return ops.linear(x, w, out=out, peer=peer)

    def reduce_norm(self, k: int, h_own: torch.Tensor, w: torch.Tensor, eps: float, Tp: int,
                    has_partial: bool, wait: bool = True) -> torch.Tensor:
        """One event: sum the partials of the owned rows into the residual, RMSNorm, gather.
        ``wait=False`` leaves the wait for the gathered rows to the consumer
        (:meth:`linear_ag`)."""
        from .. import ops
        C = _native.C()
        status = ops.ctx(self.device).status
        pushed = has_partial and self.push
        # pull mode: the reduce kernel opens the epoch and publishes this rank's partials
        # itself; push mode: the peer-output GEMM did both
        C.sp_reduce_norm_gather(self.bases, self.rank, h_own, w, float(eps),
                                self._off("p", k) if has_partial else -1, self._off("x", k), status, pushed,
                                not pushed)
        if wait:
            C.sp_wait(self.bases, self.rank, status)
        return self.gathered(k, Tp)

    def linear_ag(self, x: torch.Tensor, w):
        """Column-parallel GEMM on rows gathered by ``reduce_norm(..., wait=False)``: a
        weight-only decode GEMM waits for the gather inside the kernel (its weight stream
        starts at once); any other GEMM runs after a separate wait kernel."""
        from .. import ops
        if getattr(w, "waits_in_kernel", None) is not None and w.waits_in_kernel(x.shape[0]):
            return w.linear(x, agwait=[self.ptr, self.world])
        _native.C().sp_wait(self.bases, self.rank, ops.ctx(self.device).status)
        return ops.linear(x, w)

    def close(self):
        C = _native.C()
        for p in self._opened:
            C.symm_close(p)
        self._opened = []
        if self.ptr:
            C.symm_free(self.ptr)
            self.ptr = 0


class EmulatedSP(_SPBase):
    """Same interface over torch.distributed collectives (gloo / NCCL), no peer mapping."""

    def __init__(self, group, device, max_rows: int, dim: int, dtype=torch.float32):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device(device)
        self.max_rows = max_rows
        self.dim = dim
        self._p = [torch.zeros(max_rows, dim, dtype=dtype, device=device) for _ in range(2)]
        self._x = [torch.zeros(max_rows, dim, dtype=dtype, device=device) for _ in range(2)]

    def partial(self, k: int, rows: int) -> torch.Tensor:
        return self._p[k & 1][:rows]

    def gathered(self, k: int, rows: int) -> torch.Tensor:
        return self._x[k & 1][:rows]

    def linear_rs(self, x: torch.Tensor, w, k: int, Tp: int):
        from .. import ops
        return ops.linear(x, w, out=self.partial(k, Tp)[:x.shape[0]])

    def linear_ag(self, x: torch.Tensor, w):
        from .. import ops
        return ops.linear(x, w)

    def reduce_norm(self, k: int, h_own: torch.Tensor, w: torch.Tensor, eps: float, Tp: int,
                    has_partial: bool, wait: bool = True) -> torch.Tensor:
        own = self.own_slice(Tp)
        if has_partial:
            full = self._p[k & 1][:Tp].clone()
            if self.world > 1:
                dist.all_reduce(full, group=self.group)
            h_own.add_(full[own].to(h_own.dtype))
        x_own = ref.rmsnorm(h_own, w, eps).to(self._x[0].dtype).contiguous()
        out = self._x[k & 1][:Tp]
        if self.world > 1:
            dist.all_gather_into_tensor(out, x_own, group=self.group)
        else:
            out.copy_(x_own)
        return out

    def close(self):
        pass


def make_sp(par, device, max_rows: int, dim: int, dtype=torch.bfloat16, push: bool = False):
    """The sequence-parallel transport for this tensor-parallel group (None when tp == 1)."""
    if par.tp == 1:
        return None
    dev = torch.device(device)
    if dev.type == "cuda":
        return SymmetricSP(par.tp_group, dev, max_rows, dim, push=push)
    return EmulatedSP(par.tp_group, dev, max_rows, dim, dtype)
