"""GRPO on CPU with a small MoE policy: advantage / KL / clip math, rollout
through the engine with routing + sampling-mask capture, replay consistency,
and a parameter update that moves the reward in the right direction."""
import pytest
import torch

from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.models.config import ModelConfig, MoEConfig
from openmini_v1_b200.models.llama import DecoderLM
from openmini_v1_b200.models.policy import Policy, token_logprobs
from openmini_v1_b200.rl.grpo import GRPOConfig, group_relative_advantage, k3_kl, ppo_clip_loss
from openmini_v1_b200.rl.replay import KeepRouting, KeepSamplingMask, EnforceMode, unpack_words
from openmini_v1_b200.rl.reward import SubsetFractionReward
from openmini_v1_b200.rl.trainer import GRPOTrainer


def small_moe():
    return ModelConfig(name="moe-small", vocab_size=300, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2,
                       head_dim=16, intermediate_size=64, max_position=512, dtype="float32",
                       moe=MoEConfig(num_experts=4, top_k=2, expert_ffn=32, layer_rule="all"))


def test_grpo_math():
    r = torch.tensor([1.0, 0.0, 0.5, 0.5, 2.0, 2.0, 2.0, 2.0])
    a = group_relative_advantage(r, 4)
    assert torch.allclose(a[:4], (r[:4] - 0.5) / torch.sqrt(torch.tensor(0.125) + 1e-8))
    assert torch.allclose(a[4:], torch.zeros(4))
    lp = torch.log(torch.tensor([0.5, 0.25]))
    assert float(k3_kl(lp, lp)) == 0.0
    d = torch.tensor([0.3])
    assert abs(float(k3_kl(torch.zeros(1), d)) - float(torch.exp(d) - 1 - d)) < 1e-7
    adv = torch.tensor([1.0, -1.0])
    new, old = torch.log(torch.tensor([0.9, 0.9])), torch.log(torch.tensor([0.5, 0.5]))
    # ratio 1.8 clipped to 1.2 for the positive advantage, unclipped for the negative one
    loss = ppo_clip_loss(new, old, adv, None, 0.2)
    assert abs(float(loss) - ((-1.2) + 1.8) / 2) < 1e-5


def test_replay_caches():
    kr = KeepRouting(2, EnforceMode.STRICT)
    kr.save_routing("a", {0: torch.tensor([[1, 2]])})
    assert kr.apply_routing("a", n_tokens=1)[0].tolist() == [[1, 2]]
    kr.save_routing("b", {0: torch.tensor([[0, 1]])})
    kr.save_routing("c", {0: torch.tensor([[0, 1]])})
    assert kr.get_routing("a") is None  # evicted
    km = KeepSamplingMask()
    words = torch.tensor([[0b101]], dtype=torch.int32)
    km.save("x", words)
    out = km.apply("x", torch.zeros(1, 3))
    assert torch.isinf(out[0, 1]) and out[0, 0] == 0 and out[0, 2] == 0
    # file round trip (rollout worker -> trainer process)
    import os
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        kr.save_file(os.path.join(d, "r.pt"))
        km.save_file(os.path.join(d, "m.pt"))
        kr2, km2 = KeepRouting(4, EnforceMode.STRICT), KeepSamplingMask()
        assert kr2.load_file(os.path.join(d, "r.pt")) == 2 and km2.load_file(os.path.join(d, "m.pt")) == 1
        assert kr2.apply_routing("c", n_tokens=1)[0].tolist() == [[0, 1]]
        assert torch.equal(km2.apply("x", torch.zeros(1, 3)), out)
        torch.save({"x": 1}, os.path.join(d, "bad.pt"))
        with pytest.raises(ValueError):
            kr2.load_file(os.path.join(d, "bad.pt"))


def test_rollout_replay_and_update():
    cfg = small_moe()
    pol = Policy(cfg, seed=1)
    inf = DecoderLM(cfg, device="cpu", materialize=False)
    inf.layers = [{} for _ in range(cfg.num_layers)]
    eng = LLMEngine(inf, EngineConfig(max_num_seqs=16, max_model_len=128, enable_prefix_cache=False))
    reward = SubsetFractionReward(cfg.vocab_size, size=60, seed=3)
    tr = GRPOTrainer(pol, eng, reward, GRPOConfig(learning_rate=3e-3, group_size=4, kl_coef=0.0),
                     max_new_tokens=12, temperature=1.0, top_p=0.9)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (10,), generator=g).tolist() for _ in range(2)]
    samples = tr.rollout(prompts)
    assert len(samples) == 8
    s = samples[0]
    assert tr.keep_routing.get_routing(s["key"])[0].shape == (len(s["prompt"]) + len(s["completion"]) - 1, 2)
    # replayed forward (routing forced, no mask, T=1) reproduces the rollout's log-probs
    seq = s["prompt"] + s["completion"]
    ids = torch.tensor(seq[:-1])[None]
    logits = pol(ids, forced_routing=tr.keep_routing.apply_routing(s["key"], n_tokens=ids.shape[1]))[0]
    P = len(s["prompt"])
    lp = token_logprobs(logits[P - 1:], torch.tensor(s["completion"]))
    assert torch.allclose(lp, torch.tensor(s["rollout_logp"]), atol=2e-3), (lp, s["rollout_logp"])
    # every sampled token lies inside its recorded kept set
    words, n = tr.keep_mask.get(s["key"])
    keep = unpack_words(words, cfg.vocab_size)
    assert all(bool(keep[i, t]) for i, t in enumerate(s["completion"]))
    stats = [tr.train_step(prompts) for _ in range(6)]
    assert all(st["tokens"] > 0 for st in stats)
    assert stats[-1]["reward_mean"] > stats[0]["reward_mean"], [st["reward_mean"] for st in stats]


def _trainer(seed_offset=0, dp_group=None, train_batch=16):
    cfg = small_moe()
    pol = Policy(cfg, seed=1)
    inf = DecoderLM(cfg, device="cpu", materialize=False)
    inf.layers = [{} for _ in range(cfg.num_layers)]
    eng = LLMEngine(inf, EngineConfig(max_num_seqs=16, max_model_len=128, enable_prefix_cache=False))
    reward = SubsetFractionReward(cfg.vocab_size, size=60, seed=3)
    return GRPOTrainer(pol, eng, reward, GRPOConfig(learning_rate=3e-3, group_size=4, kl_coef=0.04),
                       max_new_tokens=8, temperature=1.0, top_p=0.9, dp_group=dp_group, train_batch=train_batch,
                       seed_offset=seed_offset)


def _prompts():
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 300, (10,), generator=g).tolist() for _ in range(2)]


def test_batched_logp_equals_per_sample():
    tr = _trainer()
    samples = tr.rollout(_prompts())
    tr.train_batch = 1
    one = tr._batch_logp(tr.policy, samples)
    tr.train_batch = 8
    many = tr._batch_logp(tr.policy, samples)
    for a, b in zip(one, many):
        assert torch.allclose(a, b, atol=1e-5)


def _dp_worker(rank, port, q):
    import os
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    tr = _trainer(seed_offset=rank, dp_group=dist.group.WORLD)
    tr.train_step([_prompts()[rank]])
    q.put((rank, {n: p.grad.numpy().copy() for n, p in tr.policy.named_parameters() if p.grad is not None}))
    dist.barrier()
    dist.destroy_process_group()


def test_data_parallel_step_matches_single_process():
    """Two gloo ranks with one prompt each (overlapped bucket all-reduce) end the step
    with the gradients of one process that trains on both prompts (the reduced, clipped
    gradients the optimizer used; Adam's first step is about lr * sign(g), which would
    turn summation-order noise of near-zero entries into lr-sized parameter differences)."""
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_dp_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(60)
    single = _trainer()
    single.train_step(_prompts())
    want = {n: p.grad for n, p in single.policy.named_parameters() if p.grad is not None}
    for r in (0, 1):
        assert res[r].keys() == want.keys()
        for n, t in res[r].items():
            scale = float(want[n].abs().max()) + 1e-12
            assert torch.allclose(torch.from_numpy(t), want[n], atol=1e-4 * scale), (r, n)
