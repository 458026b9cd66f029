"""GRPO trainer: rollout through the serving engine, replay, policy update.

One ``train_step(prompts)``:
  1. rollout: every prompt is sampled ``group_size`` times by the paged-KV
     engine (top-p sampling); the engine records each sampled token's kept set
     (Keep Sampling Mask) and every MoE layer's expert ids (Keep Routing);
  2. rewards -> group-relative advantages;
  3. batched training forward (right-padded groups of ``train_batch`` samples) of
     the fp32-master policy over prompt + completion with
     the rollout's routing forced and the rollout's kept sets applied to the
     logits; old log-probs are the same forward before the update, reference
     log-probs come from a frozen copy of the initial policy;
  4. GRPO loss (PPO clip + K3 KL), backward with the data-parallel gradient
     all-reduce started per bucket from backward hooks (``train.ddp.GradReducer``,
     overlapped with the rest of backward), clip, AdamW on fp32 masters;
  5. the new weights are pushed into the rollout model.

Reference flow: GRPOTrainer::train_step / GRPOOptimizer::train_step
(openmini-server/src/rl/actor.rs:224, grpo.rs:315-434) whose update was a
no-op; TrainingPipeline::grpo_train_step (training/pipeline.rs:872).
"""
from __future__ import annotations

import copy
import time

import torch
import torch.distributed as dist

from ..engine.request import SamplingParams
from ..models.policy import Policy, token_logprobs
from .grpo import GRPOConfig, group_relative_advantage, grpo_loss
from .replay import KeepRouting, KeepSamplingMask, unpack_words


class GRPOTrainer:
    def __init__(self, policy: Policy, engine, reward_fn, cfg: GRPOConfig | None = None, max_new_tokens: int = 64,
                 temperature: float = 1.0, top_p: float = 0.9, dp_group=None, ref_policy: Policy | None = None,
                 train_batch: int = 16, seed_offset: int = 0):
        self.policy = policy
        self.engine = engine
        self.reward_fn = reward_fn
        self.cfg = cfg or GRPOConfig()
        self.max_new = max_new_tokens
        self.temperature = temperature
        self.top_p = top_p
        self.dp_group = dp_group
        self.train_batch = train_batch
        self.seed_offset = seed_offset  # global index of this rank's first sample (data parallel)
        from ..train.ddp import GradReducer
        # gradient all-reduce in buckets, started from backward hooks as buckets complete
        self.reducer = GradReducer(policy.parameters(), group=dp_group) \
            if dp_group is not None and dist.is_initialized() and dist.get_world_size(dp_group) > 1 else None
        self.ref = ref_policy or copy.deepcopy(policy).requires_grad_(False)
        self.opt = torch.optim.AdamW(policy.parameters(), lr=self.cfg.learning_rate, betas=(0.9, 0.999),
                                     weight_decay=0.0)
        self.keep_routing = KeepRouting(10000)
        self.keep_mask = KeepSamplingMask(10000)
        self.step_idx = 0
        self.policy.export_to(self.engine.model)

    # ------------------------------------------------------------ rollout
    def rollout(self, prompts):
        moe = any(getattr(L, "is_moe", False) for L in self.policy.layers)
        sp = [SamplingParams(temperature=self.temperature, top_p=self.top_p, max_tokens=self.max_new,
                             ignore_eos=True, logprobs=True, return_sampling_mask=True, return_routing=moe,
                             seed=hash((self.step_idx, self.seed_offset + i, j)) & 0x7FFFFFFF)
              for i in range(len(prompts)) for j in range(self.cfg.group_size)]
        flat = [p for p in prompts for _ in range(self.cfg.group_size)]
        reqs = self.engine.generate(flat, sp)
        samples = []
        for k, r in enumerate(reqs):
            key = f"s{self.step_idx}-{k}"
            if r.routing:
                self.keep_routing.save_routing(key, {l: torch.cat(v) for l, v in r.routing.items()})
            if r.sampling_masks:
                self.keep_mask.save(key, torch.stack(r.sampling_masks))
            samples.append({"key": key, "prompt": r.prompt_token_ids, "completion": list(r.output_token_ids),
                            "rollout_logp": list(r.output_logprobs)})
        return samples

    # ------------------------------------------------------------ training
    def _batch_logp(self, model, samples, forced=True):
        """Per-sample completion log-probs under ``model`` with replayed routing / masks, in
        forwards of ``train_batch`` right-padded sequences (causal attention: padding after
        a sequence does not change its rows)."""
        out = []
        dev = self.policy.device
        V = self.policy.cfg.vocab_size
        for b0 in range(0, len(samples), self.train_batch):
            grp = samples[b0:b0 + self.train_batch]
            seqs = [s["prompt"] + s["completion"] for s in grp]
            T = max(len(x) for x in seqs) - 1
            ids = torch.zeros(len(grp), T, dtype=torch.long)
            for i, x in enumerate(seqs):
                ids[i, :len(x) - 1] = torch.tensor(x[:-1])
            routing = None
            if forced:
                per = [self.keep_routing.apply_routing(s["key"], dev, len(x) - 1) for s, x in zip(grp, seqs)]
                if all(r is not None for r in per) and per:
                    routing = {}
                    for layer in per[0]:
                        k = per[0][layer].shape[1]
                        rows = torch.zeros(len(grp), T, k, dtype=per[0][layer].dtype, device=dev)
                        for i, r in enumerate(per):
                            rows[i, :r[layer].shape[0]] = r[layer]
                        routing[layer] = rows.view(len(grp) * T, k)
            logits = model(ids.to(dev), forced_routing=routing)
            for i, s in enumerate(grp):
                P, C = len(s["prompt"]), len(s["completion"])
                lg = logits[i, P - 1:P - 1 + C]
                tgt = torch.tensor(s["completion"], device=dev)
                item = self.keep_mask.get(s["key"])
                keep = unpack_words(item[0][:C].to(dev), V) if item is not None else None
                out.append(token_logprobs(lg, tgt, self.temperature, keep))
        return out

    def train_step(self, prompts) -> dict:
        t0 = time.time()
        samples = self.rollout(prompts)
        t_roll = time.time() - t0
        rewards = torch.tensor([self.reward_fn(s["prompt"], s["completion"]) for s in samples], dtype=torch.float32)
        adv = group_relative_advantage(rewards, self.cfg.group_size, self.cfg.epsilon)
        with torch.no_grad():
            old = [x.detach() for x in self._batch_logp(self.policy, samples)]
            ref = [x.detach() for x in self._batch_logp(self.ref, samples)]
        self.opt.zero_grad(set_to_none=True)
        logp = self._batch_logp(self.policy, samples)
        lengths = [len(x) for x in logp]
        dev = self.policy.device
        cat = torch.cat(logp)
        adv_tok = torch.cat([torch.full((n,), float(a), device=dev) for n, a in zip(lengths, adv)])
        mask = torch.ones_like(cat, dtype=torch.bool)
        loss, stats = grpo_loss(cat, torch.cat(old), torch.cat(ref), adv_tok, mask, self.cfg)
        if self.reducer is not None:
            self.reducer.begin(last_micro_batch=True)
        loss.backward()
        if self.reducer is not None:
            self.reducer.finish()
        gn = torch.nn.utils.clip_grad_norm_(self.policy.parameters(), self.cfg.max_grad_norm)
        self.opt.step()
        self.policy.export_to(self.engine.model)
        self.step_idx += 1
        stats.update({"reward_mean": float(rewards.mean()), "grad_norm": float(gn), "rollout_s": t_roll,
                      "step_s": time.time() - t0, "samples": len(samples),
                      "completion_tokens": int(sum(lengths))})
        return stats
