"""Speculative decoding beyond greedy: the sampled acceptance rule reproduces the
sampler's distribution exactly (checked on fixed logits by counting), sampled
requests run through the engine with speculation and repeat under the same seed,
and the per-request draft length adapts to the acceptance rate."""
from types import SimpleNamespace

import torch

from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.engine.speculative import _probs, _verify_sampled
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM


def test_sampled_acceptance_preserves_the_distribution():
    V, N = 7, 20000
    logits = torch.tensor([[2.0, 1.5, 0.3, -1.0, 0.9, 0.0, -2.0],
                           [0.1, 0.4, 2.2, 1.0, -0.5, 0.8, 0.0],
                           [1.0, 1.0, 1.0, 0.0, 0.0, 0.0, 0.0]])
    params = SimpleNamespace(temperature=0.8, top_k=5, top_p=0.95, seed=None)
    eng = SimpleNamespace(cfg=SimpleNamespace(seed=3))
    p0, p1 = _probs(logits[0], params), _probs(logits[1], params)
    assert float(p0[6]) == 0.0 and float(p0.sum()) > 0.999      # top-k removed the smallest
    for draft in ([4, 2], [0, 5], [6, 3]):                      # a likely, a common and an impossible draft
        first = torch.zeros(V)
        second = torch.zeros(V)
        n_second = 0
        for t in range(N):
            r = SimpleNamespace(params=params, seq_id=1, rng_offset=t)
            out = _verify_sampled(eng, r, draft, logits)
            first[out[0]] += 1
            if out[0] == draft[0]:
                second[out[1]] += 1
                n_second += 1
        assert (first / N - p0).abs().max() < 0.015, (draft, first / N, p0)
        if n_second > 2000:
            assert (second / n_second - p1).abs().max() < 0.03, (draft, second / n_second, p1)
    # the same (seed, offset) gives the same tokens
    r = SimpleNamespace(params=params, seq_id=1, rng_offset=5)
    assert _verify_sampled(eng, r, [4, 2], logits) == _verify_sampled(eng, r, [4, 2], logits)


def test_sampled_requests_speculate_through_the_engine():
    m = DecoderLM(tiny(), device="cpu", seed=4)
    pat = [11, 12, 13, 14, 15, 16, 17, 18] * 4
    sp = SamplingParams(temperature=0.05, max_tokens=20, ignore_eos=True, seed=7)
    runs = []
    for _ in range(2):
        e = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256, speculative_k=4))
        runs.append([r.output_token_ids for r in e.generate([pat, pat[:13]], sp)])
        assert e.stats["spec_proposed"] > 0 and e.stats["spec_accepted"] > 0
    assert runs[0] == runs[1] and all(len(o) == 20 for o in runs[0])
    # at a near-zero temperature (random-init logits differ by ~1e-2) the sampled output
    # through speculation is the greedy one
    greedy = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256)).generate(
        [pat, pat[:13]], SamplingParams(temperature=0.0, max_tokens=20, ignore_eos=True))
    e = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256, speculative_k=4))
    cold = e.generate([pat, pat[:13]], SamplingParams(temperature=1e-4, max_tokens=20, ignore_eos=True, seed=1))
    assert [r.output_token_ids for r in cold] == [r.output_token_ids for r in greedy]
    assert e.stats["spec_accepted"] > 0


class _Recorder:
    """Wraps a proposer and records the draft length asked for."""

    def __init__(self, inner, k):
        self.inner, self.k, self.asked = inner, k, []

    def propose(self, toks, k=None):
        self.asked.append(k)
        return self.inner(toks, k)


def test_adaptive_draft_length():
    m = DecoderLM(tiny(), device="cpu", seed=4)
    pat = [11, 12, 13, 14, 15, 16, 17, 18] * 4
    sp = SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=True)
    cfg = EngineConfig(max_num_seqs=1, max_model_len=256, speculative_k=4, speculative_k_min=1)
    # drafts that are never the model's choice: k falls to the minimum
    e = LLMEngine(m, cfg)
    bad = _Recorder(lambda toks, k: [(toks[-1] * 7 + 3 + j) % 100 + 20000 for j in range(k)], 4)
    e.spec = bad
    base = LLMEngine(m, EngineConfig(max_num_seqs=1, max_model_len=256)).generate([pat], sp)[0].output_token_ids
    assert e.generate([pat], sp)[0].output_token_ids == base
    assert bad.asked[:5] == [4, 3, 2, 1, 1] and max(bad.asked[3:]) == 1  # (0 once max_tokens leaves no room)
    # drafts that are always right (the model's own greedy continuation): k stays at the maximum
    e2 = LLMEngine(m, cfg)
    own = LLMEngine(m, EngineConfig(max_num_seqs=1, max_model_len=256))
    good = _Recorder(lambda toks, k: list(own.generate([list(toks)], SamplingParams(
        temperature=0.0, max_tokens=k, ignore_eos=True))[0].output_token_ids) if k > 0 else [], 4)
    e2.spec = good
    assert e2.generate([pat], sp)[0].output_token_ids == base
    full = [k for k in good.asked if k is not None]
    assert full[0] == 4 and all(k == 4 for k in full[:4])
    # adaptation off: the configured k is asked for every time it fits
    e3 = LLMEngine(m, EngineConfig(max_num_seqs=1, max_model_len=256, speculative_k=4, speculative_adaptive=False))
    bad3 = _Recorder(bad.inner, 4)
    e3.spec = bad3
    e3.generate([pat], sp)
    assert bad3.asked[:5] == [4] * 5


def test_typical_acceptance_rule():
    """Typical acceptance keeps a draft whose probability clears min(epsilon, delta e^-H)
    and rejects one below it; on rejection the token comes from the full distribution."""
    import math
    logits = torch.tensor([[3.0, 2.0, 0.0, -1.0], [0.0, 0.0, 0.0, 0.0], [1.0, 0.0, 0.0, 0.0]])
    params = SimpleNamespace(temperature=1.0, top_k=0, top_p=1.0, seed=None)
    cfg = SimpleNamespace(seed=0, speculative_acceptance="typical", typical_epsilon=0.09, typical_delta=0.3)
    eng = SimpleNamespace(cfg=cfg)
    p0 = _probs(logits[0], params)
    ent = float(-(p0 * p0.log()).sum())
    thr = min(0.09, 0.3 * math.exp(-ent))
    assert float(p0[1]) > thr > float(p0[3])
    r = SimpleNamespace(params=params, seq_id=1, rng_offset=0)
    out = _verify_sampled(eng, r, [1, 2], logits)      # p1 uniform over 4: 0.25 > min(0.09, 0.3/4)
    assert out[:2] == [1, 2] and len(out) == 3
    counts = torch.zeros(4)
    for t in range(4000):
        o = _verify_sampled(eng, SimpleNamespace(params=params, seq_id=1, rng_offset=t), [3], logits)
        assert len(o) == 1                                # the unlikely draft is always rejected
        counts[o[0]] += 1
    assert (counts / 4000 - p0).abs().max() < 0.03
    cfg.speculative_acceptance = "bogus"
    import pytest
    with pytest.raises(ValueError):
        _verify_sampled(eng, r, [1], logits)
