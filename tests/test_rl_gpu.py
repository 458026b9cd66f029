"""GRPO on the GPU with a small MoE policy: rollout through the CUDA engine with
routing / sampling-mask capture, replayed log-probs, and one update step."""
import pytest
import torch

from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.models.config import ModelConfig, MoEConfig
from openmini_v1_b200.models.llama import DecoderLM
from openmini_v1_b200.models.policy import Policy
from openmini_v1_b200.rl.grpo import GRPOConfig
from openmini_v1_b200.rl.reward import SubsetFractionReward
from openmini_v1_b200.rl.trainer import GRPOTrainer

pytestmark = pytest.mark.gpu


def test_grpo_step_on_gpu():
    cfg = ModelConfig(name="moe-gpu", vocab_size=512, hidden_size=256, num_layers=2, num_heads=2, num_kv_heads=1,
                      head_dim=128, intermediate_size=256, max_position=512,
                      moe=MoEConfig(num_experts=4, top_k=2, expert_ffn=128, layer_rule="all"))
    pol = Policy(cfg, device="cuda", seed=1)
    inf = DecoderLM(cfg, device="cuda", materialize=False)
    inf.layers = [{} for _ in range(cfg.num_layers)]
    eng = LLMEngine(inf, EngineConfig(max_num_seqs=8, max_model_len=128, enable_prefix_cache=False,
                                      use_cuda_graph=False))
    tr = GRPOTrainer(pol, eng, SubsetFractionReward(cfg.vocab_size, size=100, seed=3),
                     GRPOConfig(learning_rate=1e-3, group_size=4, kl_coef=0.04), max_new_tokens=8,
                     temperature=1.0, top_p=0.9)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (12,), generator=g).tolist() for _ in range(2)]
    before = pol.lm_head.detach().clone()
    st = tr.train_step(prompts)
    assert st["completion_tokens"] > 0 and all(torch.isfinite(torch.tensor(float(v))) for v in st.values())
    assert not torch.equal(before, pol.lm_head.detach())
