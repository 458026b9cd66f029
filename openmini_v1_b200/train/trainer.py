"""Supervised trainer (causal LM / SFT) with gradient accumulation, LR schedule,
gradient clipping, data-parallel gradient reduction overlapped with backward,
periodic checkpoints with resume, evaluation with early stopping, and
pause / resume / stop control for the training REST API.

The model is the trainable :class:`~openmini_v1_b200.models.policy.Policy`
(fp32 masters, bf16 tcgen05 GEMMs on the GPU). Unlike the reference, whose
forward is a mock returning random logits (openmini-server/src/training/
trainer.rs:770), the loss here is the model's real next-token cross entropy.

Reference: Trainer::train / train_step / evaluate / early stopping / pause,
resume, stop (openmini-server/src/training/trainer.rs:42-1190), TrainingConfig
field names kept.
"""
from __future__ import annotations

import dataclasses
import threading
import time
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from .checkpoint import CheckpointManager
from .ddp import GradReducer
from .loss import DynamicLossScaler, causal_lm_loss, perplexity
from .optim import make_optimizer, make_schedule, set_lr


@dataclass
class TrainingConfig:
    mode: str = "causal_lm"              # "causal_lm" | "sft" (SFT masks prompt labels in the dataset)
    num_train_epochs: int = 3
    per_device_train_batch_size: int = 8
    gradient_accumulation_steps: int = 1
    learning_rate: float = 1e-4
    weight_decay: float = 0.01
    adam_beta1: float = 0.9
    adam_beta2: float = 0.999
    adam_epsilon: float = 1e-8
    max_grad_norm: float = 1.0
    max_seq_length: int = 2048
    label_smoothing_factor: float = 0.0
    output_dir: str = "./checkpoints"
    save_steps: int = 500
    save_total_limit: int = 5
    logging_steps: int = 10
    early_stopping_patience: int = 5
    early_stopping_threshold: float = 0.001
    lr_scheduler: str = "cosine"         # cosine | linear | constant
    warmup_steps: int = 0
    min_lr: float = 0.0
    optimizer: str = "adamw"
    fp16_loss_scaling: bool = False
    seed: int = 0
    max_steps: int = 0                   # 0: run all epochs


@dataclass
class TrainingState:
    epoch: int = 0
    global_step: int = 0
    micro_step: int = 0
    best_eval_loss: float | None = None
    epochs_without_improvement: int = 0
    status: str = "idle"                 # idle | running | paused | stopped | finished | early_stopped
    last_loss: float | None = None
    lr: float = 0.0
    history: list = field(default_factory=list)


class Trainer:
    def __init__(self, model, cfg: TrainingConfig, train_loader, eval_loader=None, dp_group=None, log=None):
        self.model, self.cfg = model, cfg
        self.train_loader, self.eval_loader = train_loader, eval_loader
        self.device = next(model.parameters()).device
        self.opt = make_optimizer(model, cfg.optimizer, cfg.learning_rate, cfg.weight_decay,
                                  (cfg.adam_beta1, cfg.adam_beta2), cfg.adam_epsilon)
        steps_per_epoch = max(1, len(train_loader) // cfg.gradient_accumulation_steps)
        total = cfg.max_steps or steps_per_epoch * cfg.num_train_epochs
        self.total_steps = total
        self.sched = make_schedule(cfg.lr_scheduler, cfg.learning_rate, cfg.warmup_steps, total, cfg.min_lr)
        self.scaler = DynamicLossScaler(enabled=cfg.fp16_loss_scaling)
        self.reducer = GradReducer(model.parameters(), dp_group)
        self.ckpt = CheckpointManager(cfg.output_dir, cfg.save_total_limit)
        self.state = TrainingState()
        self.rank = dist.get_rank(dp_group) if dist.is_initialized() else 0
        self.log = log or (lambda *a, **k: None)
        self._run = threading.Event()
        self._run.set()
        self._stop = False

    # ------------------------------------------------------------ control
    def pause(self):
        if self.state.status == "running":
            self._run.clear()
            self.state.status = "paused"

    def resume(self):
        if self.state.status == "paused":
            self.state.status = "running"
            self._run.set()

    def stop(self):
        self._stop = True
        self._run.set()

    def status(self) -> dict:
        s = dataclasses.asdict(self.state)
        s["history"] = s["history"][-50:]
        s["total_steps"] = self.total_steps
        return s

    # ------------------------------------------------------------ steps
    def _loss(self, batch):
        ids = batch["input_ids"].to(self.device)
        labels = batch["labels"].to(self.device)
        logits = self.model(ids)
        return causal_lm_loss(logits, labels, self.cfg.label_smoothing_factor)

    def _optimizer_step(self) -> dict:
        self.reducer.finish()
        params = [p for p in self.model.parameters() if p.grad is not None]
        ok = self.scaler.unscale_and_check(params)
        gn = float(torch.nn.utils.clip_grad_norm_(params, self.cfg.max_grad_norm)) if params else 0.0
        lr = self.sched.get_lr(self.state.global_step)
        set_lr(self.opt, lr)
        if ok:
            self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        self.state.global_step += 1
        self.state.lr = lr
        return {"grad_norm": gn, "lr": lr, "skipped": not ok}

    @torch.no_grad()
    def evaluate(self) -> float | None:
        if self.eval_loader is None:
            return None
        self.model.eval()
        tot, n = 0.0, 0
        for batch in self.eval_loader:
            tot += float(self._loss(batch))
            n += 1
        self.model.train()
        t = torch.tensor([tot, float(n)], device=self.device)
        if dist.is_initialized() and self.reducer.world > 1:
            dist.all_reduce(t, group=self.reducer.group)
        return float(t[0] / t[1].clamp(min=1))

    def save(self, val_loss=None) -> str | None:
        if self.rank != 0:
            return None
        st = dataclasses.asdict(self.state)
        st["history"] = st["history"][-200:]
        st["config"] = dataclasses.asdict(self.cfg)
        return self.ckpt.save(self.model, self.opt, st, {"scaler": self.scaler.state_dict()}, val_loss)

    def resume_from_checkpoint(self, path: str | None = None) -> bool:
        p = path or self.ckpt.latest()
        if p is None:
            return False
        st = self.ckpt.load(p, self.model, self.opt)
        for k in ("epoch", "global_step", "micro_step", "best_eval_loss", "epochs_without_improvement"):
            setattr(self.state, k, st.get(k, getattr(self.state, k)))
        self.scaler.load_state_dict(st["extra"].get("scaler", self.scaler.state_dict()))
        return True

    def train(self) -> TrainingState:
        cfg, st = self.cfg, self.state
        st.status = "running"
        self.model.train()
        acc = cfg.gradient_accumulation_steps
        start_epoch = st.epoch
        for epoch in range(start_epoch, cfg.num_train_epochs):
            st.epoch = epoch
            self.train_loader.set_epoch(epoch)
            skip = st.micro_step if epoch == start_epoch else 0  # resume inside an epoch
            t0 = time.time()
            for i, batch in enumerate(self.train_loader):
                if i < skip:
                    continue
                self._run.wait()
                if self._stop:
                    st.status = "stopped"
                    return st
                last = (i + 1) % acc == 0
                self.reducer.begin(last)
                loss = self._loss(batch)
                self.scaler.scale_loss(loss / acc).backward()
                st.micro_step = i + 1
                st.last_loss = float(loss.detach())
                if not last:
                    continue
                info = self._optimizer_step()
                if st.global_step % cfg.logging_steps == 0:
                    rec = {"step": st.global_step, "epoch": epoch, "loss": st.last_loss, **info,
                           "s_per_step": (time.time() - t0) / cfg.logging_steps}
                    st.history.append(rec)
                    self.log("train", **rec)
                    t0 = time.time()
                if cfg.save_steps and st.global_step % cfg.save_steps == 0:
                    self.save()
                if cfg.max_steps and st.global_step >= cfg.max_steps:
                    st.status = "finished"
                    self.save(self.evaluate())
                    return st
            st.micro_step = 0
            ev = self.evaluate()
            if ev is not None:
                self.log("eval", epoch=epoch, loss=ev, ppl=perplexity(ev))
                st.history.append({"step": st.global_step, "epoch": epoch, "eval_loss": ev})
                if st.best_eval_loss is None or st.best_eval_loss - ev > cfg.early_stopping_threshold:
                    st.best_eval_loss = ev
                    st.epochs_without_improvement = 0
                else:
                    st.epochs_without_improvement += 1
                st.epoch = epoch + 1
                self.save(ev)
                if st.epochs_without_improvement >= cfg.early_stopping_patience:
                    st.status = "early_stopped"
                    return st
            else:
                st.epoch = epoch + 1
        st.status = "finished"
        return st
