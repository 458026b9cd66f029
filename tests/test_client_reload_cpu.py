"""Synchronous gRPC client (channel pool, retries) against the OpenMini service on
CPU, and hot model reload: a request migrated to the standby engine mid-generation
finishes with the same greedy tokens as an uninterrupted run."""
import asyncio
import threading

import grpc
import pytest

from openmini_v1_b200.engine.async_engine import AsyncLLMEngine
from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.engine.tokenizer import ByteTokenizer
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM


def _engine(seed=0):
    return LLMEngine(DecoderLM(tiny(), device="cpu", seed=seed), EngineConfig(max_num_seqs=4, max_model_len=256))


def test_sync_client_against_grpc_server():
    from openmini_v1_b200.client import OpenMiniClient
    from openmini_v1_b200.serve.grpc_server import OpenMiniServicer, start_grpc_server
    aeng = AsyncLLMEngine(_engine())
    tok = ByteTokenizer()
    loop = asyncio.new_event_loop()
    started = threading.Event()
    box = {}

    def serve():
        asyncio.set_event_loop(loop)
        server, port = loop.run_until_complete(start_grpc_server(OpenMiniServicer(aeng, tok), "127.0.0.1:0"))
        box["server"], box["port"] = server, port
        started.set()
        loop.run_forever()

    th = threading.Thread(target=serve, daemon=True)
    th.start()
    assert started.wait(30)
    try:
        with OpenMiniClient(f"127.0.0.1:{box['port']}", pool_size=2, timeout_s=60) as c:
            assert c.health_check()
            r = c.chat([("user", "hello")], session_id="s1", max_tokens=6)
            assert r.completion_tokens == 6 and r.session_id == "s1" and len(r.tokens) == 5
            r2 = c.chat([("user", "hello")], session_id="s2", max_tokens=6, stream=False)
            assert r2.text == r.text  # greedy, same prompt
            toks = list(c.chat_stream([("user", "x")], max_tokens=3))
            assert toks[-1].finished and toks[-1].usage.completion_tokens == 3
            with pytest.raises(grpc.RpcError) as e:
                c.image_understanding(b"\x89PNG", "what?")
            assert e.value.code() == grpc.StatusCode.UNIMPLEMENTED
            assert c.stats["errors"] == 1
        # an unreachable server: retries then reports unhealthy
        with OpenMiniClient("127.0.0.1:1", timeout_s=0.5, max_retries=1, backoff_s=0.01) as bad:
            assert not bad.health_check()
            assert bad.stats["retries"] == 1
    finally:
        loop.call_soon_threadsafe(loop.stop)
        th.join(10)
        aeng.shutdown()


def test_hot_reload_migrates_requests():
    from openmini_v1_b200.serve.hot_reload import HotReloader
    prompt = list(range(40, 60))
    sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True)
    want = _engine().generate([prompt], sp)[0].output_token_ids
    hr = HotReloader(_engine(), name="v1")
    eng = hr.engine()
    req = eng.add_request("r0", prompt, SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True))
    for _ in range(5):
        eng.step()
    assert 0 < len(req.output_token_ids) < 12
    hr.preload_standby(lambda: _engine(seed=0), name="v2")
    assert hr.wait_standby(60)
    st = hr.status()
    assert st["standby_ready"] and st["standby"]["name"] == "v2"
    assert hr.switch_to_standby(migrate=True) == 2
    new = hr.engine()
    assert new is not eng and not eng.has_unfinished()
    while new.has_unfinished():
        new.step()
    assert req.output_token_ids == want
    assert hr.rollback() == 1 and hr.engine() is eng
    # a failing loader is reported, the active engine is untouched
    hr.release_standby()
    hr.preload_standby(lambda: (_ for _ in ()).throw(RuntimeError("bad checkpoint")), name="v3")
    assert not hr.wait_standby(10)
    assert "bad checkpoint" in hr.status()["error"] and hr.engine() is eng
