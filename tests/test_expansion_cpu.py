"""Function-preserving model growth (depth, width, heads, FFN) and the phased
pretrain -> SFT -> GRPO pipeline."""
import pytest
import torch

from openmini_v1_b200.models.config import ModelConfig
from openmini_v1_b200.models.policy import Policy
from openmini_v1_b200.train.expansion import PipelineConfig, PhaseConfig, TrainingPipeline, expand_policy


def _cfg(**kw):
    d = dict(name="b", vocab_size=300, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=16,
             intermediate_size=128, max_position=256, dtype="float32")
    d.update(kw)
    return ModelConfig(**d)


def test_expansion_preserves_function_and_trains():
    base = Policy(_cfg(), seed=1)
    big = expand_policy(base, _cfg(hidden_size=96, num_heads=6, num_kv_heads=3, intermediate_size=192, num_layers=4))
    ids = torch.randint(0, 300, (2, 20), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        a, b = base(ids), big(ids)
    assert (a - b).abs().max() < 1e-5 * a.abs().max()
    n_big = sum(p.numel() for p in big.parameters())
    assert n_big > 2 * sum(p.numel() for p in base.parameters())
    loss = torch.nn.functional.cross_entropy(big(ids[:, :-1]).reshape(-1, 300), ids[:, 1:].reshape(-1))
    loss.backward()
    o3 = dict(big.named_parameters())["layers.3.o"]
    assert o3.grad.abs().sum() > 0  # the identity block's output projection learns
    rnd = expand_policy(base, _cfg(hidden_size=96, num_heads=6, num_kv_heads=3, intermediate_size=192),
                        strategy="random")
    with torch.no_grad():
        assert (rnd(ids) - a).abs().max() > 1e-3
    with pytest.raises(ValueError):
        expand_policy(base, _cfg(num_heads=8, num_kv_heads=2))  # GQA ratio changes


def test_phased_pipeline():
    pol = Policy(_cfg(), seed=2)
    pipe = TrainingPipeline(pol, PipelineConfig(pretrain=PhaseConfig(3e-3, 10, 2), sft=PhaseConfig(1e-3, 5, 0)))
    ids = torch.randint(0, 300, (4, 24), generator=torch.Generator().manual_seed(1))
    losses = [pipe.step(ids)["loss"] for _ in range(10)]
    assert losses[-1] < losses[0] and pipe.log[0]["lr"] < pipe.log[1]["lr"]  # warm-up
    pipe.switch_phase("sft")
    mask = torch.zeros_like(ids, dtype=torch.bool)
    mask[:, 12:] = True  # only response tokens count
    out = pipe.step((ids, mask))
    assert out["phase"] == "sft" and out["step"] == 0 and abs(out["lr"] - 1e-3) < 1e-9
    with pytest.raises(ValueError):
        pipe.switch_phase("grpo")
