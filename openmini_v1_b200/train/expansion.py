"""Model growth (e.g. 7B -> 14B) and the phased training pipeline around it.

``expand_policy(base, target_cfg)`` builds a larger dense ``Policy`` whose initial
function equals the base model's exactly:

* depth: the target's layers are spread over the base layers (target layer j copies
  base layer floor(j L / L')'s weights when it is the first copy; every further copy
  is a new block whose output projections o and down are zero, so it adds nothing to
  the residual until training moves them);
* width: every old weight sits in the top-left block of the new matrix; new rows that
  feed only new features (q / k / v rows of new heads, gate / up rows of new FFN
  features) are small random, every entry through which a new feature could reach
  an old one (new columns of o, down and the embedding, new rows of o and down) is
  zero, so the new hidden dimensions stay exactly zero in the forward;
* RMSNorm: with the hidden size going from D to D' and the new dimensions zero, the
  root mean square shrinks by sqrt(D / D'); the old norm weights are multiplied by
  that factor and the RMSNorm epsilon by D / D' (then S / D' + eps D / D' =
  (D / D') (S / D + eps) for the sum of squares S), which restores every normalised
  activation exactly.
New query heads keep the base's GQA ratio (head h reads KV head h // G in both
models). ``strategy="random"`` instead initialises the new parts randomly
(function not preserved), and ``"scaled_copy"`` copies layers without the zero
output projections (a depth up-scaling).

``TrainingPipeline`` runs the phases pretrain -> SFT -> GRPO with one optimizer per
phase (learning rate, warm-up and cosine schedule of the phase) and reports the
phase of every step.

Reference counterparts: openmini-server/src/training/pipeline.rs:439-500
(expand_from_checkpoint with RandomInit / ScaledCopy / Interpolation; there it pads a
flat parameter vector), :763-806 (switch_phase), training/config.rs (Model14BConfig,
TrainingConfig14B).
"""
from __future__ import annotations

import copy
import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from ..models.config import ModelConfig
from ..models.policy import Policy


def _grow(old: torch.Tensor, shape, rows_rand=None, std=0.02, gen=None, zero=True):
    """New tensor of ``shape`` with ``old`` in the top-left block; the rest zero, except
    rows ``rows_rand`` (a slice or index list of new rows), filled N(0, std)."""
    out = torch.zeros(shape, dtype=old.dtype, device=old.device)
    if not zero:
        out.normal_(0.0, std, generator=gen)
    if rows_rand is not None:
        r = torch.randn(out[rows_rand].shape, generator=gen) * std
        out[rows_rand] = r.to(out.dtype)
    out[tuple(slice(0, s) for s in old.shape)] = old
    return out


def _qkv_rows(cfg: ModelConfig):
    H, Hk, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    return slice(0, H * hd), slice(H * hd, (H + Hk) * hd), slice((H + Hk) * hd, (H + 2 * Hk) * hd)


@torch.no_grad()
def expand_policy(base: Policy, target: ModelConfig, strategy: str = "preserve", seed: int = 0) -> Policy:
    b = base.cfg
    if b.moe.num_experts or target.moe.num_experts:
        raise ValueError("expansion supports dense FFN layers")
    if target.head_dim != b.head_dim or target.num_heads * b.num_kv_heads != b.num_heads * target.num_kv_heads:
        raise ValueError("keep head_dim and the query / KV head ratio")
    if (target.hidden_size < b.hidden_size or target.num_heads < b.num_heads
            or target.intermediate_size < b.intermediate_size or target.num_layers < b.num_layers
            or target.vocab_size != b.vocab_size):
        raise ValueError("the target must be at least as large in every dimension, same vocabulary")
    g = torch.Generator().manual_seed(seed)
    D, D2 = b.hidden_size, target.hidden_size
    zero = strategy != "random"
    if zero:
        target = copy.deepcopy(target)
        target.rms_eps = b.rms_eps * D / D2
    new = Policy(target, device="cpu", seed=seed)
    norm_scale = math.sqrt(D / D2) if zero else 1.0
    bp = {n: p.detach().float().cpu() for n, p in base.named_parameters()}
    sd = {}
    sd["embed"] = _grow(bp["embed"], (target.vocab_size, D2), gen=g, zero=zero)
    sd["lm_head"] = _grow(bp["lm_head"], (target.vocab_size, D2), gen=g, zero=zero)
    sd["norm"] = torch.cat([bp["norm"] * norm_scale, torch.ones(D2 - D) * (1.0 if not zero else norm_scale)])
    L, L2 = b.num_layers, target.num_layers
    first_copy = {}
    for j in range(L2):
        src = j * L // L2
        extra = src in first_copy  # a further copy of this base layer
        first_copy.setdefault(src, j)
        pre = f"layers.{src}."
        H, Hk, hd = b.num_heads, b.num_kv_heads, b.head_dim
        H2, Hk2 = target.num_heads, target.num_kv_heads
        qkv = bp[pre + "qkv"]
        (q0, k0, v0), (q1, k1, v1) = _qkv_rows(b), _qkv_rows(target)
        parts = []
        for o_sl, n_old, n_new in ((q0, H * hd, H2 * hd), (k0, Hk * hd, Hk2 * hd), (v0, Hk * hd, Hk2 * hd)):
            parts.append(_grow(qkv[o_sl], (n_new, D2), rows_rand=slice(n_old, n_new), gen=g, zero=zero))
        sd[f"layers.{j}.qkv"] = torch.cat(parts)
        o = _grow(bp[pre + "o"], (D2, H2 * hd), gen=g, zero=zero)
        F1, F2 = b.intermediate_size, target.intermediate_size
        gu = bp[pre + "gate_up"]
        gate = _grow(gu[:F1], (F2, D2), rows_rand=slice(F1, F2), gen=g, zero=zero)
        up = _grow(gu[F1:], (F2, D2), rows_rand=slice(F1, F2), gen=g, zero=zero)
        down = _grow(bp[pre + "down"], (D2, F2), gen=g, zero=zero)
        if extra and strategy == "preserve":  # a further copy starts as an identity block
            o.zero_()
            down.zero_()
        sd[f"layers.{j}.o"], sd[f"layers.{j}.gate_up"], sd[f"layers.{j}.down"] = o, torch.cat([gate, up]), down
        for nm in ("attn_norm", "ffn_norm"):
            w = bp[pre + nm]
            sd[f"layers.{j}.{nm}"] = torch.cat([w * norm_scale, torch.full((D2 - D,), norm_scale if zero else 1.0)])
    new.load_state_dict(sd, strict=False)
    return new.to(base.device) if base.device.type != "cpu" else new


# ----------------------------------------------------------------------------- phased pipeline

@dataclass
class PhaseConfig:
    lr: float
    steps: int
    warmup: int = 0
    weight_decay: float = 0.01
    min_lr_ratio: float = 0.1


@dataclass
class PipelineConfig:
    pretrain: PhaseConfig = field(default_factory=lambda: PhaseConfig(3e-4, 100, 10))
    sft: PhaseConfig = field(default_factory=lambda: PhaseConfig(5e-5, 50, 5))
    grpo: PhaseConfig = field(default_factory=lambda: PhaseConfig(1e-6, 20, 0, 0.0))


PHASES = ("pretrain", "sft", "grpo")


class TrainingPipeline:
    def __init__(self, policy: Policy, cfg: PipelineConfig | None = None, grpo_trainer=None):
        self.policy, self.cfg = policy, cfg or PipelineConfig()
        self.grpo = grpo_trainer
        self.phase = None
        self.step_in_phase = 0
        self.log: list[dict] = []
        self.switch_phase("pretrain")

    def switch_phase(self, phase: str):
        if phase not in PHASES:
            raise ValueError(f"unknown phase {phase!r}")
        if phase == "grpo" and self.grpo is None:
            raise ValueError("the GRPO phase needs a GRPOTrainer")
        pc = getattr(self.cfg, phase)
        self.opt = torch.optim.AdamW(self.policy.parameters(), lr=pc.lr, weight_decay=pc.weight_decay)
        if phase == "grpo":
            self.grpo.opt = self.opt
        self.phase, self.step_in_phase = phase, 0

    def lr(self) -> float:
        pc = getattr(self.cfg, self.phase)
        s = self.step_in_phase
        if s < pc.warmup:
            return pc.lr * (s + 1) / pc.warmup
        t = (s - pc.warmup) / max(1, pc.steps - pc.warmup)
        return pc.lr * (pc.min_lr_ratio + (1 - pc.min_lr_ratio) * 0.5 * (1 + math.cos(math.pi * min(t, 1.0))))

    def _lm_step(self, ids: torch.Tensor, loss_mask: torch.Tensor | None):
        for grp in self.opt.param_groups:
            grp["lr"] = self.lr()
        logits = self.policy(ids[:, :-1].to(self.policy.device))
        tgt = ids[:, 1:].to(logits.device)
        loss = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1), reduction="none")
        m = loss_mask[:, 1:].to(logits.device).reshape(-1).float() if loss_mask is not None else torch.ones_like(loss)
        loss = (loss * m).sum() / m.sum().clamp(min=1)
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(self.policy.parameters(), 1.0)
        self.opt.step()
        return float(loss.detach())

    def step(self, batch) -> dict:
        """pretrain: token ids [B, T]; sft: (ids [B, T], response mask [B, T]); grpo: prompts."""
        if self.phase == "pretrain":
            out = {"loss": self._lm_step(batch, None)}
        elif self.phase == "sft":
            ids, mask = batch
            out = {"loss": self._lm_step(ids, mask)}
        else:
            out = self.grpo.train_step(batch)
        out.update(phase=self.phase, step=self.step_in_phase, lr=self.lr())
        self.step_in_phase += 1
        self.log.append(out)
        return out
