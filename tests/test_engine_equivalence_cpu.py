"""Greedy outputs do not depend on scheduling (hypothesis over prompt sets): the
same requests give the same tokens with whole or chunked prefill under any token
budget, with the prefix cache on or off, under a KV pool small enough to force
preemption (recompute or swap), and with n-gram speculative decoding (also under KV
pressure) -- as one request at a time with plenty of memory."""
import random

from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM

MODEL = DecoderLM(tiny(), device="cpu", seed=21)


def _run(prompts, outs, **kw):
    cfg = dict(max_num_seqs=4, max_model_len=192, use_cuda_graph=False)
    cfg.update(kw)
    eng = LLMEngine(MODEL, EngineConfig(**cfg))
    res = eng.generate(prompts, [SamplingParams(temperature=0.0, max_tokens=n, ignore_eos=True) for n in outs])
    return [r.output_token_ids for r in res], eng.stats


@settings(max_examples=6, deadline=None)
@given(seed=st.integers(0, 10 ** 6), n=st.integers(2, 5))
def test_greedy_outputs_independent_of_scheduling(seed, n):
    rng = random.Random(seed)
    shared = [rng.randrange(300, 30000) for _ in range(24)]
    prompts = [shared[:rng.randrange(0, 24)] + [rng.randrange(300, 30000) for _ in range(rng.randrange(1, 40))]
               for _ in range(n)]
    outs = [rng.randrange(1, 30) for _ in range(n)]
    want = [_run([p], [o], max_num_seqs=1, enable_prefix_cache=False)[0][0] for p, o in zip(prompts, outs)]
    for kw in ({}, {"max_num_batched_tokens": 7}, {"enable_chunked_prefill": False},
               {"enable_prefix_cache": False}, {"num_blocks": 10}, {"num_blocks": 10, "preemption_mode": "swap"},
               {"num_blocks": 10, "max_num_batched_tokens": 16}, {"speculative_k": 3},
               {"speculative_k": 4, "num_blocks": 10}):
        got, stats = _run(prompts, outs, **kw)
        assert got == want, kw
