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


def test_attention_autograd_matches_fp32():
    import math
    from openmini_v1_b200.ops import autograd as ag
    g = torch.Generator(device="cuda").manual_seed(0)
    B, T, H, Hkv, D = 2, 200, 8, 2, 128
    mk = lambda *s: (torch.randn(*s, generator=g, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_(True)
    q, k, v = mk(B, T, H, D), mk(B, T, Hkv, D), mk(B, T, Hkv, D)
    go = torch.randn(B, T, H, D, generator=g, device="cuda").to(torch.bfloat16)
    out = ag.attention(q, k, v, 1 / math.sqrt(D))
    out.backward(go)
    qf, kf, vf = (x.detach().float().requires_grad_(True) for x in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(
        qf.transpose(1, 2), kf.transpose(1, 2), vf.transpose(1, 2), is_causal=True, enable_gqa=True).transpose(1, 2)
    ref.backward(go.float())
    rel = lambda a, b: float((a.float() - b).abs().max() / (b.abs().max() + 1e-9))
    assert rel(out, ref) < 2e-2
    assert rel(q.grad, qf.grad) < 3e-2 and rel(k.grad, kf.grad) < 3e-2 and rel(v.grad, vf.grad) < 3e-2


def test_policy_logits_and_grads_match_fp32():
    """The GPU policy (bf16 tcgen05 GEMMs and attention) against the same weights in fp32 on the CPU."""
    import copy
    from openmini_v1_b200.models.config import ModelConfig, MoEConfig
    from openmini_v1_b200.models.policy import Policy
    cfg = ModelConfig(name="p", vocab_size=512, hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=128, intermediate_size=512, max_position=1024, dtype="float32",
                      moe=MoEConfig(num_experts=4, top_k=2, expert_ffn=128, layer_rule="cyclic", cycle_period=2))
    cpu = Policy(cfg, device="cpu", seed=3)
    gpu = copy.deepcopy(cpu).to("cuda")
    gpu.device, gpu.cdt = torch.device("cuda"), torch.bfloat16
    gpu.inv_freq = gpu.inv_freq.to("cuda")
    ids = torch.randint(0, 512, (2, 150), generator=torch.Generator().manual_seed(1))
    lc = cpu(ids)
    lg = gpu(ids.cuda())
    # bf16 activations through two layers: compare in norm (single entries drift more)
    assert float((lg.detach().cpu() - lc.detach()).norm() / lc.detach().norm()) < 3e-2
    tgt = torch.randint(0, 512, (2, 150), generator=torch.Generator().manual_seed(2))
    torch.nn.functional.cross_entropy(lc.view(-1, 512), tgt.view(-1)).backward()
    torch.nn.functional.cross_entropy(lg.view(-1, 512), tgt.cuda().view(-1)).backward()
    for (n, pc), (_, pg) in zip(cpu.named_parameters(), gpu.named_parameters()):
        if pc.grad is None:
            continue
        rel = float((pg.grad.cpu() - pc.grad).norm() / (pc.grad.norm() + 1e-12))
        assert rel < 0.1, (n, rel)
