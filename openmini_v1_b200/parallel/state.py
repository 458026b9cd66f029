"""Process groups for tensor / expert / data / pipeline parallelism.

One process per GPU. ``init_distributed`` reads RANK / WORLD_SIZE / LOCAL_RANK
/ MASTER_ADDR / MASTER_PORT (torchrun) and creates the NCCL (GPU) or gloo
(CPU) world group; ``ParallelState`` then carves it into a mesh
``world = pp x dp x tp`` (tp fastest, so a TP group is NVLink-adjacent ranks)
with expert-parallel groups laid over dp x tp.

Replaces the reference's configuration-only parallel layer
(openmini-server/src/distributed/config.rs:70-153 CommBackend / ranks / master
port 29500, openmini-server/src/model/inference/distributed_inference_config.rs:48-228
ParallelStrategy presets) with real process groups.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


def init_distributed(backend: str | None = None, timeout_s: float = 600.0) -> tuple[int, int]:
    """Initialise the default process group from the environment (idempotent)."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world == 1:
        return 0, 1
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29500")
    kw = {}
    if backend == "nccl":
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend=backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world


@dataclass
class ParallelState:
    rank: int = 0
    world: int = 1
    tp: int = 1
    dp: int = 1
    pp: int = 1
    ep: int = 1
    tp_group: object = None
    dp_group: object = None
    pp_group: object = None
    ep_group: object = None
    tp_rank: int = 0
    dp_rank: int = 0
    pp_rank: int = 0
    ep_rank: int = 0

    @staticmethod
    def single() -> "ParallelState":
        return ParallelState()

    @staticmethod
    def build(tp: int = 1, pp: int = 1, ep: int = 1) -> "ParallelState":
        if not (dist.is_available() and dist.is_initialized()):
            if tp * pp * ep != 1:
                raise RuntimeError("torch.distributed must be initialised for tp/pp/ep > 1")
            return ParallelState.single()
        rank, world = dist.get_rank(), dist.get_world_size()
        if world % (tp * pp) != 0:
            raise ValueError(f"world {world} not divisible by tp*pp={tp * pp}")
        dp = world // (tp * pp)
        if (dp * tp) % ep != 0:
            raise ValueError(f"ep {ep} must divide dp*tp={dp * tp}")
        st = ParallelState(rank=rank, world=world, tp=tp, dp=dp, pp=pp, ep=ep)
        # rank = ((pp_i * dp) + dp_i) * tp + tp_i ; every rank creates every group (collective)
        for p in range(pp):
            for d in range(dp):
                ranks = [(p * dp + d) * tp + t for t in range(tp)]
                g = (dist.new_group(ranks) if tp < world else dist.group.WORLD) if tp > 1 else None
                if rank in ranks:
                    st.tp_group, st.tp_rank = g, ranks.index(rank)
            for t in range(tp):
                ranks = [(p * dp + d) * tp + t for d in range(dp)]
                g = (dist.new_group(ranks) if dp < world else dist.group.WORLD) if dp > 1 else None
                if rank in ranks:
                    st.dp_group, st.dp_rank = g, ranks.index(rank)
            stage = [(p * dp + d) * tp + t for d in range(dp) for t in range(tp)]
            for j in range(0, len(stage), ep):
                ranks = stage[j:j + ep]
                g = (dist.new_group(ranks) if ep < world else dist.group.WORLD) if ep > 1 else None
                if rank in ranks:
                    st.ep_group, st.ep_rank = g, ranks.index(rank)
        for d in range(dp):
            for t in range(tp):
                ranks = [(p * dp + d) * tp + t for p in range(pp)]
                g = (dist.new_group(ranks) if pp < world else dist.group.WORLD) if pp > 1 else None
                if rank in ranks:
                    st.pp_group, st.pp_rank = g, ranks.index(rank)
        return st
