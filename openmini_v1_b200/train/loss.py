"""Training losses and loss scaling.

``causal_lm_loss``: next-token cross entropy over positions whose label is not
``ignore_index`` (prompt tokens of SFT samples are masked that way), with
optional label smoothing (reference: openmini-server/src/training/loss.rs:6-280).

``DynamicLossScaler``: fp16 training scales the loss, skips a step whose
gradients overflowed and halves the scale, and doubles it after
``growth_interval`` clean steps (reference LossScaler, training/amp.rs:10-30).
bf16 training does not need it (scale stays 1).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

IGNORE = -100


def causal_lm_loss(logits: torch.Tensor, labels: torch.Tensor, label_smoothing: float = 0.0,
                   ignore_index: int = IGNORE) -> torch.Tensor:
    """logits [B, T, V] predict labels [B, T] shifted by one: position t predicts labels[t + 1]."""
    lg = logits[:, :-1].reshape(-1, logits.shape[-1]).float()
    tgt = labels[:, 1:].reshape(-1)
    if not bool((tgt != ignore_index).any()):
        return lg.sum() * 0.0
    return F.cross_entropy(lg, tgt, ignore_index=ignore_index, label_smoothing=label_smoothing)


def perplexity(loss: float) -> float:
    import math
    return math.exp(min(loss, 50.0))


class DynamicLossScaler:
    def __init__(self, init_scale: float = 2.0 ** 16, growth_factor: float = 2.0, backoff_factor: float = 0.5,
                 growth_interval: int = 2000, enabled: bool = True):
        self.scale = float(init_scale) if enabled else 1.0
        self.growth_factor, self.backoff_factor = growth_factor, backoff_factor
        self.growth_interval = growth_interval
        self.enabled = enabled
        self._good = 0
        self.skipped = 0

    def scale_loss(self, loss: torch.Tensor) -> torch.Tensor:
        return loss * self.scale if self.enabled else loss

    def unscale_and_check(self, params) -> bool:
        """Divide gradients by the scale; False (and back off) if any is inf / nan."""
        if not self.enabled:
            return True
        grads = [p.grad for p in params if p.grad is not None]
        finite = True
        for g in grads:
            g.div_(self.scale)
            if not bool(torch.isfinite(g).all()):
                finite = False
        if finite:
            self._good += 1
            if self._good >= self.growth_interval:
                self.scale *= self.growth_factor
                self._good = 0
        else:
            self.scale = max(self.scale * self.backoff_factor, 1.0)
            self._good = 0
            self.skipped += 1
        return finite

    def state_dict(self):
        return {"scale": self.scale, "good": self._good, "skipped": self.skipped}

    def load_state_dict(self, s):
        self.scale, self._good, self.skipped = s["scale"], s["good"], s["skipped"]
