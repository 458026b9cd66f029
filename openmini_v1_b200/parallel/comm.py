"""Collective operations.

``CollectiveOps`` keeps the reference's interface
(openmini-server/src/distributed/communication.rs:85-177: all_reduce with
Sum/Max/Min/Prod/Avg, all_gather, reduce_scatter, broadcast, barrier) but runs
on torch.distributed process groups: NCCL over NVLink on GPUs, gloo on CPU.
It is the baseline transport for the tensor-parallel layers.

``LocalComm`` is the in-process N-rank fake used by the reference's tests
(communication.rs:209-527): ranks are objects sharing one buffer table, which
keeps single-process unit tests of TP math possible.
"""
from __future__ import annotations

import enum
import threading

import torch
import torch.distributed as dist


class ReduceOp(enum.Enum):
    SUM = "sum"
    MAX = "max"
    MIN = "min"
    PROD = "prod"
    AVG = "avg"


_TORCH_OP = {ReduceOp.SUM: "SUM", ReduceOp.MAX: "MAX", ReduceOp.MIN: "MIN", ReduceOp.PROD: "PRODUCT"}


class CollectiveOps:
    """Collectives over a torch.distributed group (None = world)."""

    def __init__(self, group=None):
        self.group = group
        self.enabled = dist.is_available() and dist.is_initialized()
        self.size = dist.get_world_size(group) if self.enabled else 1
        self.rank = dist.get_rank(group) if self.enabled else 0

    def all_reduce(self, t: torch.Tensor, op: ReduceOp = ReduceOp.SUM) -> torch.Tensor:
        if self.size == 1:
            return t
        if op == ReduceOp.AVG:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            t.div_(self.size)
            return t
        dist.all_reduce(t, op=getattr(dist.ReduceOp, _TORCH_OP[op]), group=self.group)
        return t

    def all_gather(self, t: torch.Tensor, dim: int = -1) -> torch.Tensor:
        if self.size == 1:
            return t
        t = t.contiguous()
        flat = torch.empty((self.size * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(flat, t, group=self.group)
        out = flat.view((self.size,) + tuple(t.shape))
        dim = dim % t.dim()
        if dim == 0:
            return out.reshape((-1,) + tuple(t.shape[1:]))
        return torch.cat(list(out.unbind(0)), dim=dim)

    def reduce_scatter(self, t: torch.Tensor, dim: int = 0) -> torch.Tensor:
        if self.size == 1:
            return t
        if dim != 0:
            t = t.movedim(dim, 0)
        t = t.contiguous()
        out = torch.empty((t.shape[0] // self.size,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.reduce_scatter_tensor(out, t, group=self.group)
        return out.movedim(0, dim) if dim != 0 else out

    def broadcast(self, t: torch.Tensor, root: int = 0) -> torch.Tensor:
        if self.size == 1:
            return t
        src = dist.get_global_rank(self.group, root) if self.group is not None else root
        dist.broadcast(t, src=src, group=self.group)
        return t

    def barrier(self):
        if self.size > 1:
            dist.barrier(group=self.group)

    def all_to_all(self, t: torch.Tensor, in_splits=None, out_splits=None) -> torch.Tensor:
        if self.size == 1:
            return t
        t = t.contiguous()  # before empty_like, so the output is dense whatever t's strides were
        if in_splits is None:
            out = torch.empty_like(t)
            dist.all_to_all_single(out, t, group=self.group)
            return out
        out = torch.empty((sum(out_splits),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_to_all_single(out, t, out_splits, in_splits, group=self.group)
        return out


class _LocalShared:
    def __init__(self, n):
        self.n = n
        self.slots = [None] * n
        self.cv = threading.Condition()
        self.gen = 0
        self.arrived = 0
        self.result = None


class LocalComm:
    """In-process collectives for N rank objects driven from N threads."""

    def __init__(self, rank: int, shared: _LocalShared):
        self.rank, self.shared, self.size = rank, shared, shared.n

    @staticmethod
    def create(n: int) -> list:
        sh = _LocalShared(n)
        return [LocalComm(r, sh) for r in range(n)]

    def _exchange(self, value, combine, timeout=30.0):
        sh = self.shared
        with sh.cv:
            gen = sh.gen
            sh.slots[self.rank] = value
            sh.arrived += 1
            if sh.arrived == sh.n:
                sh.result = combine(list(sh.slots))
                sh.arrived = 0
                sh.gen += 1
                sh.cv.notify_all()
            elif not sh.cv.wait_for(lambda: sh.gen != gen, timeout=timeout):
                raise TimeoutError("LocalComm: peers did not arrive")
            return sh.result

    def all_reduce(self, t: torch.Tensor, op: ReduceOp = ReduceOp.SUM) -> torch.Tensor:
        def comb(xs):
            s = torch.stack([x.float() for x in xs])
            return {ReduceOp.SUM: lambda: s.sum(0), ReduceOp.AVG: lambda: s.mean(0),
                    ReduceOp.MAX: lambda: s.max(0).values, ReduceOp.MIN: lambda: s.min(0).values,
                    ReduceOp.PROD: lambda: s.prod(0)}[op]()
        r = self._exchange(t.clone(), comb)
        t.copy_(r.to(t.dtype))
        return t

    def all_gather(self, t: torch.Tensor, dim: int = -1) -> torch.Tensor:
        return self._exchange(t.clone(), lambda xs: torch.cat(xs, dim=dim)).clone()

    def reduce_scatter(self, t: torch.Tensor, dim: int = 0) -> torch.Tensor:
        r = self._exchange(t.clone(), lambda xs: torch.stack([x.float() for x in xs]).sum(0))
        return r.chunk(self.size, dim=dim)[self.rank].to(t.dtype).clone()

    def broadcast(self, t: torch.Tensor, root: int = 0) -> torch.Tensor:
        r = self._exchange(t.clone(), lambda xs: xs[root])
        t.copy_(r)
        return t

    def barrier(self):
        self._exchange(None, lambda xs: None)


# ----------------------------------------------------------------------------- backends + failover

BACKENDS: dict = {}


def register_backend(name: str, factory):
    """``factory(**kw) -> object with the CollectiveOps interface``."""
    BACKENDS[name] = factory


def make_backend(name: str, **kw):
    if name not in BACKENDS:
        raise KeyError(f"unknown communication backend {name!r}; registered: {sorted(BACKENDS)}")
    return BACKENDS[name](**kw)


register_backend("nccl", lambda group=None: CollectiveOps(group))   # process group of the NCCL backend
register_backend("gloo", lambda group=None: CollectiveOps(group))   # a gloo process group (CPU / control)
register_backend("local", lambda rank, shared: LocalComm(rank, shared))


class FailoverComm:
    """Collectives over a primary backend that fall back to a secondary one (for example
    NCCL over NVLink -> gloo over TCP) once the primary raises; the switch is sticky and
    recorded. Every rank must fail over together, which holds when the primary fails on
    all of them (a dead link or process group); ``on_failover(name, exc)`` lets the
    caller notify the cluster control plane.

    Reference counterpart: openmini-server/src/distributed/exo_communication.rs
    (backend selection with failover between transports)."""

    OPS = ("all_reduce", "all_gather", "reduce_scatter", "broadcast", "barrier", "all_to_all")

    def __init__(self, primary, secondary, on_failover=None, names=("primary", "secondary")):
        self.backends = [primary, secondary]
        self.names = names
        self.active = 0
        self.failures: list = []
        self.on_failover = on_failover

    def _call(self, op, *a, **kw):
        try:
            return getattr(self.backends[self.active], op)(*a, **kw)
        except Exception as e:
            if self.active == 1:
                raise
            self.failures.append((op, repr(e)))
            self.active = 1
            if self.on_failover:
                self.on_failover(self.names[1], e)
            return getattr(self.backends[1], op)(*a, **kw)

    def __getattr__(self, op):
        if op in FailoverComm.OPS:
            return lambda *a, **kw: self._call(op, *a, **kw)
        raise AttributeError(op)

    @property
    def backend_name(self) -> str:
        return self.names[self.active]
