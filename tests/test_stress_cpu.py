"""Stress, leak and concurrency checks on CPU (the reference's stress_test.rs,
memory_leak_test.rs and concurrent_stress_test.rs, as real engine work):

* request churn with aborts mid-prefill and mid-decode, preemption under a small KV
  pool and the prefix cache on: after every round all KV blocks are free again and
  the engine holds no request;
* many concurrent async streams, some cancelled by their consumer: every stream ends
  and nothing is left in flight;
* repeated rounds do not grow the engine's bookkeeping."""
import asyncio
import random

import pytest
import torch

from openmini_v1_b200.engine.async_engine import AsyncLLMEngine
from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM


def _engine(num_blocks=None, prefix=True, **kw):
    m = DecoderLM(tiny(), device="cpu", seed=11)
    cfg = EngineConfig(max_num_seqs=6, max_model_len=160, enable_prefix_cache=prefix, use_cuda_graph=False,
                       num_blocks=num_blocks, **kw)
    return LLMEngine(m, cfg)


@pytest.mark.parametrize("kw", [{}, {"preemption_mode": "swap"}, {"speculative_k": 3}],
                         ids=["recompute", "swap", "speculative"])
def test_churn_with_aborts_and_preemption_frees_every_block(kw):
    eng = _engine(num_blocks=14, **kw)
    free0 = eng.bm.num_free()
    rng = random.Random(3)
    shared = [rng.randrange(300, 30000) for _ in range(40)]
    sizes = []
    for rnd in range(4):
        ids = []
        for i in range(10):
            prompt = (shared[:rng.randrange(0, 40)] + [rng.randrange(300, 30000) for _ in range(rng.randrange(3, 50))])
            rid = f"r{rnd}-{i}"
            eng.add_request(rid, prompt, SamplingParams(temperature=rng.choice([0.0, 0.8]),
                                                        max_tokens=rng.randrange(1, 70), ignore_eos=True))
            ids.append(rid)
        steps = 0
        while eng.has_unfinished():
            eng.step()
            steps += 1
            if steps in (1, 3, 7):  # abort one request early (prefill) and some later (decode)
                victim = rng.choice(ids)
                eng.abort_request(victim)
            assert steps < 2000
        assert eng.bm.num_free() == free0, (rnd, eng.bm.num_free(), free0)
        assert not eng.requests
        sizes.append(len(eng.stats))
    assert sizes[-1] == sizes[1]  # no per-round growth of the bookkeeping
    assert eng.bm.num_blocks == 14 and eng.stats["preemptions"] > 0  # the small pool forced preemption


def test_concurrent_async_streams_with_cancellation():
    eng = _engine()
    free0 = eng.bm.num_free()
    aeng = AsyncLLMEngine(eng)
    try:
        async def consume(i):
            sp = SamplingParams(temperature=0.0, max_tokens=8 + i % 5, ignore_eos=True)
            n = 0
            async for out in aeng.generate([100 + i, 200 + i, 300 + i] * (1 + i % 4), sp):
                n += 1
                if i % 4 == 3 and n == 2:  # the consumer walks away mid-stream
                    return -1
            return n

        async def main():
            return await asyncio.wait_for(asyncio.gather(*(consume(i) for i in range(24))), timeout=120)
        res = asyncio.run(main())
        for i, n in enumerate(res):
            assert n == (-1 if i % 4 == 3 else 8 + i % 5), (i, n)
        deadline = 0
        while (eng.has_unfinished() or eng.requests) and deadline < 200:  # aborts land on the engine thread
            import time
            time.sleep(0.01)
            deadline += 1
        assert not eng.requests and eng.bm.num_free() == free0
    finally:
        aeng.shutdown()


def test_http_completions_under_concurrent_clients():
    """24 clients at once through the HTTP API (plain and SSE streaming): every answer
    has the requested length and the engine ends with nothing in flight."""
    from concurrent.futures import ThreadPoolExecutor

    from fastapi.testclient import TestClient

    from openmini_v1_b200.engine.tokenizer import ByteTokenizer
    from openmini_v1_b200.serve.http import create_app
    eng = _engine()
    free0 = eng.bm.num_free()
    aeng = AsyncLLMEngine(eng)
    try:
        with TestClient(create_app(aeng, ByteTokenizer(), "tiny")) as c:
            def call(i):
                body = {"prompt": [300 + i, 301 + i, 302 + i] * (1 + i % 3), "max_tokens": 4 + i % 4,
                        "temperature": 0.0, "ignore_eos": True}
                if i % 2:
                    r = c.post("/v1/completions", json=dict(body, stream=True))
                    events = [ln for ln in r.text.splitlines() if ln.startswith("data: ") and ln != "data: [DONE]"]
                    return r.status_code, len(events)
                r = c.post("/v1/completions", json=body)
                return r.status_code, r.json()["usage"]["completion_tokens"]
            with ThreadPoolExecutor(12) as ex:
                res = list(ex.map(call, range(24)))
        assert res == [(200, 4 + i % 4) for i in range(24)], res
        import time
        for _ in range(200):
            if not eng.requests:
                break
            time.sleep(0.01)
        assert not eng.requests and eng.bm.num_free() == free0
    finally:
        aeng.shutdown()
