"""Optimizers and learning-rate schedules of the trainer.

Schedules follow the reference's definitions
(openmini-server/src/training/optimizer.rs:441-560): linear warmup from 0 to the
target rate over ``warmup_steps``, then cosine decay to ``min_lr`` over the
remaining steps (CosineWithWarmup), linear decay to ``min_lr`` (LinearWithWarmup)
or a constant rate.

AdamW keeps fp32 master weights and fp32 moments (the parameters themselves are
the fp32 masters; compute runs in bf16 on the GPU). Decoupled weight decay is
not applied to 1-D parameters (norm gains).
"""
from __future__ import annotations

import math

import torch


class CosineWithWarmup:
    def __init__(self, warmup_steps: int, total_steps: int, min_lr: float, target_lr: float):
        self.warmup_steps, self.total_steps = int(warmup_steps), int(total_steps)
        self.min_lr, self.target_lr = float(min_lr), float(target_lr)

    def get_lr(self, step: int) -> float:
        if step < self.warmup_steps:
            return self.target_lr * step / max(self.warmup_steps, 1)
        progress = (step - self.warmup_steps) / max(self.total_steps - self.warmup_steps, 1)
        return self.min_lr + 0.5 * (self.target_lr - self.min_lr) * (1.0 + math.cos(math.pi * progress))


class LinearWithWarmup:
    def __init__(self, warmup_steps: int, total_steps: int, min_lr: float, target_lr: float):
        self.warmup_steps, self.total_steps = int(warmup_steps), int(total_steps)
        self.min_lr, self.target_lr = float(min_lr), float(target_lr)

    def get_lr(self, step: int) -> float:
        if step < self.warmup_steps:
            return self.target_lr * step / max(self.warmup_steps, 1)
        if step >= self.total_steps:
            return self.min_lr
        progress = (step - self.warmup_steps) / (self.total_steps - self.warmup_steps)
        return self.target_lr - (self.target_lr - self.min_lr) * progress


class ConstantLR:
    def __init__(self, lr: float):
        self.lr = float(lr)

    def get_lr(self, step: int) -> float:
        return self.lr


def make_schedule(kind: str, lr: float, warmup_steps: int, total_steps: int, min_lr: float = 0.0):
    if kind == "cosine":
        return CosineWithWarmup(warmup_steps, total_steps, min_lr, lr)
    if kind == "linear":
        return LinearWithWarmup(warmup_steps, total_steps, min_lr, lr)
    if kind == "constant":
        return ConstantLR(lr)
    raise ValueError(f"unknown lr schedule {kind!r}")


def param_groups(model: torch.nn.Module, weight_decay: float):
    decay, no_decay = [], []
    for p in model.parameters():
        if not p.requires_grad:
            continue
        (no_decay if p.dim() < 2 else decay).append(p)
    return [{"params": decay, "weight_decay": weight_decay}, {"params": no_decay, "weight_decay": 0.0}]


def make_optimizer(model, kind: str = "adamw", lr: float = 1e-4, weight_decay: float = 0.01,
                   betas=(0.9, 0.999), eps: float = 1e-8, momentum: float = 0.0):
    groups = param_groups(model, weight_decay)
    if kind == "adamw":
        return torch.optim.AdamW(groups, lr=lr, betas=betas, eps=eps)
    if kind == "sgd":
        return torch.optim.SGD(groups, lr=lr, momentum=momentum)
    raise ValueError(f"unknown optimizer {kind!r}")


def set_lr(opt, lr: float):
    for g in opt.param_groups:
        g["lr"] = lr
