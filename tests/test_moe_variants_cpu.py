"""MoE variants: shared experts, zero-computation (identity) experts, forced routing to
a zero expert, and the load-balance auxiliary loss."""
from types import SimpleNamespace

import torch

from openmini_v1_b200 import ops
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM
from openmini_v1_b200.models.moe import load_balance_loss, moe_forward


def test_shared_and_zero_experts():
    cfg = tiny()
    cfg.moe.num_experts, cfg.moe.top_k, cfg.moe.expert_ffn = 4, 2, 64
    cfg.moe.num_shared_experts, cfg.moe.num_zero_experts = 1, 2
    m = DecoderLM(cfg, device="cpu", seed=0, dtype=torch.float32)
    L = m.layers[0]
    assert L["router"].shape[0] == 6 and L["shared_gate_up"].shape[0] == 2 * 64
    x = torch.randn(5, cfg.hidden_size)
    shared = ops.linear(ops.silu_mul(ops.linear(x, L["shared_gate_up"])), L["shared_down"])
    # both choices forced onto zero experts 4 and 5: routed part is exactly x
    fb = SimpleNamespace(forced_routing={0: torch.tensor([[4, 5]] * 5)}, record_routing=None)
    y = moe_forward(m, 0, L, x, fb)
    assert torch.allclose(y, x + shared, atol=1e-5)
    # normal routing runs and mixes real and zero experts
    fb2 = SimpleNamespace(forced_routing=None, record_routing={})
    y2 = moe_forward(m, 0, L, x, fb2)
    assert y2.shape == x.shape and torch.isfinite(y2).all()
    assert int(fb2.record_routing[0].max()) < 6


def test_load_balance_loss():
    E = 4
    ids = torch.arange(8).view(4, 2) % E
    lg = torch.zeros(4, E)
    assert abs(float(load_balance_loss(lg, ids, E)) - 1.0) < 1e-6
    skew = torch.zeros(4, 2, dtype=torch.long)
    lg2 = torch.tensor([[5.0, 0, 0, 0]] * 4)
    assert float(load_balance_loss(lg2, skew, E)) > 2.0
