"""Sharded optimizer state (ZeRO stage 1/2) for data-parallel training, and the
training memory estimator.

``ShardedAdamW`` keeps fp32 master weights and the AdamW moments for only this
rank's 1/W slice of the flattened parameters. A step is

  1. reduce-scatter of the (bf16 or fp32) gradients into this rank's slice,
     averaged over the data-parallel group (stage 2: no rank holds the full
     reduced gradient),
  2. AdamW on the slice in fp32 (decoupled weight decay, bias correction),
  3. all-gather of the updated slice into every rank's model parameters.

With W ranks the optimizer memory per rank drops from 12 bytes per parameter
(fp32 master + m + v) to 12 / W. On GPUs the collectives are NCCL over NVLink
(the reduce-scatter can start as soon as the backward pass has produced the
bucket); on CPU gloo (tests).

``estimate_memory`` restates the reference's ZeRO / FSDP memory estimators
(openmini-server/src/training/distributed_config.rs:47-535: DataParallelConfig,
DeepSpeedConfig stages 0-3, FSDP sharding) for planning.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist


class ShardedAdamW:
    def __init__(self, params, lr: float = 1e-4, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.0,
                 group=None):
        self.params = [p for p in params if p.requires_grad]
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.group = group
        self.W = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.numel = sum(p.numel() for p in self.params)
        self.shard = math.ceil(self.numel / self.W)
        self.padded = self.shard * self.W
        dev = self.params[0].device
        flat = torch.zeros(self.padded, dtype=torch.float32, device=dev)
        flat[:self.numel] = torch.cat([p.detach().float().reshape(-1) for p in self.params])
        lo = self.rank * self.shard
        self.master = flat[lo:lo + self.shard].clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.t = 0

    def state_bytes(self) -> int:
        return 3 * self.master.numel() * 4

    def zero_grad(self):
        for p in self.params:
            p.grad = None

    @torch.no_grad()
    def step(self):
        dev = self.master.device
        g = torch.zeros(self.padded, dtype=torch.float32, device=dev)
        o = 0
        for p in self.params:
            n = p.numel()
            if p.grad is not None:
                g[o:o + n] = p.grad.float().reshape(-1)
            o += n
        gs = torch.empty(self.shard, dtype=torch.float32, device=dev)
        if self.W > 1:
            dist.reduce_scatter_tensor(gs, g, group=self.group)
            gs /= self.W
        else:
            gs.copy_(g)
        self.t += 1
        b1, b2 = self.betas
        self.m.mul_(b1).add_(gs, alpha=1 - b1)
        self.v.mul_(b2).addcmul_(gs, gs, value=1 - b2)
        mhat = self.m / (1 - b1 ** self.t)
        vhat = self.v / (1 - b2 ** self.t)
        self.master.mul_(1 - self.lr * self.wd)
        self.master.addcdiv_(mhat, vhat.sqrt_().add_(self.eps), value=-self.lr)
        full = torch.empty(self.padded, dtype=torch.float32, device=dev)
        if self.W > 1:
            dist.all_gather_into_tensor(full, self.master, group=self.group)
        else:
            full.copy_(self.master)
        o = 0
        for p in self.params:
            n = p.numel()
            p.copy_(full[o:o + n].view_as(p).to(p.dtype))
            o += n


@dataclass
class MemoryEstimate:
    weights_gb: float
    grads_gb: float
    optimizer_gb: float
    activations_gb: float

    @property
    def total_gb(self) -> float:
        return self.weights_gb + self.grads_gb + self.optimizer_gb + self.activations_gb


def estimate_memory(params_b: float, dp: int, zero_stage: int = 1, param_bytes: int = 2, grad_bytes: int = 2,
                    tokens_per_gpu: int = 8192, hidden: int = 4096, layers: int = 32,
                    activation_checkpointing: bool = True) -> MemoryEstimate:
    """Per-GPU training memory for ZeRO stage 0-3 (stage 3 == FSDP full sharding).

    Optimizer state is fp32 master + two AdamW moments (12 B / parameter). Activations:
    ~34 B per token per hidden unit per layer without checkpointing, ~2 B with it."""
    P = params_b * 1e9
    w = P * param_bytes / (dp if zero_stage >= 3 else 1)
    g = P * grad_bytes / (dp if zero_stage >= 2 else 1)
    o = P * 12 / (dp if zero_stage >= 1 else 1)
    per = 2 if activation_checkpointing else 34
    a = tokens_per_gpu * hidden * layers * per
    return MemoryEstimate(w / 1e9, g / 1e9, o / 1e9, a / 1e9)
