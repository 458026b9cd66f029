"""GRPO objective pieces (differentiable, token-level, masked).

Restates the math of openmini-server/src/rl/grpo.rs:19-263 and the
configuration of openmini-server/src/rl/mod.rs:140-164:

* group-relative advantage  A_i = (r_i - mean(r)) / sqrt(var(r) + eps)
* K3 KL estimator           KL = exp(d) - 1 - d, d = logp_ref - logp, masked mean
* off-policy sequence mask  drop tokens with negative advantage whose KL
                            exceeds a threshold
* PPO-clip policy loss      -min(r A, clip(r, 1-e, 1+e) A), masked mean
* total                     pg + kl_coef * KL - ent_coef * H

Two reference quirks are not reproduced (documented deviations): the
unmasked reference loss takes min() of the summed surrogates instead of the
per-token min, and its entropy of log-probabilities is identically zero
(it only counts positive log-probs); here the per-token PPO min is used and
the entropy is the exact entropy of the sampling distribution when logits are
given (else the sample estimate -E[log p]).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class GRPOConfig:
    learning_rate: float = 1e-6
    kl_coef: float = 0.04
    clip_epsilon: float = 0.2
    group_size: int = 8
    epsilon: float = 1e-8
    entropy_coef: float = 0.0
    max_grad_norm: float = 1.0
    kl_mask_threshold: float = 0.0   # 0 disables the off-policy sequence mask


def group_relative_advantage(rewards: torch.Tensor, group_size: int, eps: float = 1e-8) -> torch.Tensor:
    """rewards [num_groups * group_size] -> advantages of the same shape (population variance)."""
    r = rewards.reshape(-1, group_size).double()
    mean = r.mean(1, keepdim=True)
    var = ((r - mean) ** 2).mean(1, keepdim=True)
    return ((r - mean) / torch.sqrt(var + eps)).reshape(-1).to(rewards.dtype)


def _masked_mean(x, mask):
    if mask is None:
        return x.mean()
    m = mask.to(x.dtype)
    return (x * m).sum() / m.sum().clamp_min(1.0)


def k3_kl(logp: torch.Tensor, ref_logp: torch.Tensor, mask=None) -> torch.Tensor:
    d = (ref_logp - logp).clamp(-20, 20)
    return _masked_mean((torch.exp(d) - 1 - d).clamp(max=1e6), mask)


def off_policy_mask(logp, old_logp, advantages_tok, threshold: float):
    """1 = keep; tokens with negative advantage and K3 KL above ``threshold`` are dropped."""
    d = (logp - old_logp).detach()
    kl = (torch.exp(d) - 1 - d).abs()
    return ~((advantages_tok < 0) & (kl > threshold))


def ppo_clip_loss(logp, old_logp, advantages_tok, mask=None, clip_eps: float = 0.2):
    ratio = torch.exp(logp - old_logp)
    s1 = ratio * advantages_tok
    s2 = ratio.clamp(1 - clip_eps, 1 + clip_eps) * advantages_tok
    return _masked_mean(-torch.minimum(s1, s2), mask)


def entropy(logits=None, logp=None, mask=None):
    if logits is not None:
        lp = torch.log_softmax(logits.float(), -1)
        h = -(lp.exp() * lp).sum(-1)
        return _masked_mean(h, mask)
    return _masked_mean(-logp, mask)


def grpo_loss(logp, old_logp, ref_logp, advantages_tok, mask, cfg: GRPOConfig, logits=None):
    """Returns (total loss, stats dict). All token tensors are flat [n_tokens]."""
    m = mask.bool()
    if cfg.kl_mask_threshold > 0:
        m = m & off_policy_mask(logp, old_logp, advantages_tok, cfg.kl_mask_threshold)
    pg = ppo_clip_loss(logp, old_logp, advantages_tok, m, cfg.clip_epsilon)
    kl = k3_kl(logp, ref_logp, m) if ref_logp is not None else torch.zeros((), device=logp.device)
    ent = entropy(logits, logp, m) if cfg.entropy_coef else torch.zeros((), device=logp.device)
    total = pg + cfg.kl_coef * kl - cfg.entropy_coef * ent
    with torch.no_grad():
        ratio = torch.exp(logp - old_logp)
        clipped = ((ratio - 1).abs() > cfg.clip_epsilon).float()
        stats = {"loss": float(total), "pg_loss": float(pg), "kl": float(kl), "entropy": float(ent),
                 "clip_frac": float(_masked_mean(clipped, m)), "tokens": int(m.sum())}
    return total, stats
