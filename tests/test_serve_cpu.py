"""Serving stack on CPU with the tiny model: HTTP (OpenAI + /api/v1 routes,
SSE streaming), gRPC OpenMini service, raw-TCP gateway, worker pool (with a
worker that dies and is restarted), task scheduler / batch pool, config
loading, GGUF write -> read round trip."""
import asyncio
import json
import struct

import numpy as np
import pytest
import torch
from fastapi.testclient import TestClient

from openmini_v1_b200 import _native
from openmini_v1_b200.config.settings import ServerConfig, load_config
from openmini_v1_b200.engine.async_engine import AsyncLLMEngine
from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.engine.tokenizer import ByteTokenizer, GGUFTokenizer, IncrementalDecoder
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM, ForwardBatch
from openmini_v1_b200.serve.http import create_app


@pytest.fixture(scope="module")
def stack():
    m = DecoderLM(tiny(), device="cpu", seed=0)
    eng = LLMEngine(m, EngineConfig(max_num_seqs=4, max_model_len=256))
    aeng = AsyncLLMEngine(eng)
    tok = ByteTokenizer()
    yield aeng, tok, m
    aeng.shutdown()


def test_http_completions_and_routes(stack):
    aeng, tok, m = stack
    c = TestClient(create_app(aeng, tok, "tiny"))
    r = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 5, "temperature": 0})
    assert r.status_code == 200, r.text
    j = r.json()
    assert j["usage"]["completion_tokens"] == 5 and len(j["choices"][0]["token_ids"]) == 5
    r2 = c.post("/v1/completions", json={"prompt": tok.encode("hello"), "max_tokens": 5, "temperature": 0})
    assert r2.json()["choices"][0]["token_ids"] == j["choices"][0]["token_ids"]  # deterministic greedy
    s = c.post("/v1/completions", json={"prompt": "hi", "max_tokens": 4, "stream": True})
    events = [ln for ln in s.text.split("\n\n") if ln.startswith("data: ")]
    assert events[-1] == "data: [DONE]" and len(events) == 5
    assert c.get("/health").json()["status"] == "healthy"
    assert c.get("/api/v1/health").status_code == 200
    assert "openmini_inference_requests_total" in c.get("/metrics").text
    assert c.get("/v1/models").json()["data"][0]["id"] == "tiny"
    assert c.post("/v1/completions", json={"prompt": "x", "max_tokens": 0}).status_code == 400
    ch = c.post("/api/v1/chat", json={"message": "hey", "max_tokens": 3, "temperature": 0}).json()
    assert ch["usage"]["completion_tokens"] == 3
    comp = c.post("/api/v1/inference/compute", json={"q": [[1.0, 0.0]], "k": [[1.0, 0.0], [0.0, 1.0]],
                                                      "v": [[1.0, 2.0], [3.0, 4.0]]}).json()
    w = torch.softmax(torch.tensor([1.0, 0.0]) / 2 ** 0.5, 0)
    assert abs(comp["output"][0][0] - float(w[0] * 1 + w[1] * 3)) < 1e-5
    assert c.get("/api/v1/inference/stats").json()["engine"]["decode_tokens"] > 0
    assert c.post("/api/v1/tts", json={}).status_code == 501


def test_grpc_chat_and_health(stack):
    aeng, tok, m = stack
    from openmini_v1_b200.serve.grpc_server import OpenMiniClient, OpenMiniServicer, start_grpc_server

    async def run():
        server, port = await start_grpc_server(OpenMiniServicer(aeng, tok), "127.0.0.1:0")
        cl = OpenMiniClient(f"127.0.0.1:{port}")
        try:
            assert await cl.health()
            outs = await cl.chat([("user", "hi there")], session_id="s1", max_tokens=4, stream=True)
            assert outs[-1].finished and outs[-1].usage.completion_tokens == 4
            assert len(outs) == 4  # 3 streamed tokens + final message with usage
            outs2 = await cl.chat([("user", "again")], session_id="s1", max_tokens=2, stream=False)
            assert outs2[-1].finished and outs2[-1].usage.prompt_tokens > outs[-1].usage.prompt_tokens
        finally:
            await cl.close()
            await server.stop(1)
    asyncio.run(run())


def test_gateway_frames(stack):
    aeng, tok, m = stack
    from openmini_v1_b200.serve.gateway import Gateway
    rt = _native.rt()

    async def run():
        gw = Gateway(aeng, tok, max_tokens=3)
        port = await gw.start()
        r, w = await asyncio.open_connection("127.0.0.1", port)
        w.write(rt.encode_gateway(4, "sess", False, b""))
        await w.drain()
        n = struct.unpack(">I", await r.readexactly(4))[0]
        assert await r.readexactly(n) == b"OK"
        w.write(rt.encode_gateway(1, "sess", False, b"hello"))
        await w.drain()
        n = struct.unpack(">I", await r.readexactly(4))[0]
        await r.readexactly(n)
        w.close()
        await gw.stop()
        assert gw.stats["requests"] == 2
    asyncio.run(run())


def test_worker_pool_restart_after_crash():
    from openmini_v1_b200.serve.worker_pool import WorkerPool
    pool = WorkerPool(2, "openmini_v1_b200.serve.worker_main:crash_handler", health_check_interval_ms=200)
    try:
        assert pool.dispatch(b"abc") == (True, b"ABC")
        ok, msg = pool.dispatch(b"crash")      # the worker process dies mid-task
        assert not ok and b"failed" in msg
        import time
        deadline = time.time() + 20
        while time.time() < deadline and pool.stats()["alive"] < 2:
            time.sleep(0.1)
        assert pool.stats()["alive"] == 2 and pool.restarts >= 1
        assert pool.dispatch(b"xyz") == (True, b"XYZ")
        assert all(pool.health_check().values())
    finally:
        pool.shutdown()


def test_task_scheduler_and_batch_pool():
    from openmini_v1_b200.serve.task_scheduler import AsyncInferencePool, QueueFull, TaskScheduler

    async def run():
        s = TaskScheduler(max_concurrent=2, queue_capacity=2, task_timeout_s=0.5)
        await s.start()

        async def job(v):
            await asyncio.sleep(0.01)
            return v * 2
        futs = [s.submit(lambda v=v: job(v))[1] for v in range(2)]
        assert await asyncio.gather(*futs) == [0, 2]

        async def slow():
            await asyncio.sleep(5)
        _, f = s.submit(slow)
        with pytest.raises(TimeoutError):
            await f
        await s.shutdown()
        seen = []
        pool = AsyncInferencePool(lambda ts: seen.append(len(ts)) or [t.upper() for t in ts], batch_size=4,
                                  batch_timeout_ms=20)
        await pool.start()
        res = await asyncio.gather(*[pool.submit(c) for c in "abcdef"])
        assert res == list("ABCDEF") and max(seen) <= 4 and sum(seen) == 6
        await pool.shutdown()
    asyncio.run(run())


def test_config_semantics(tmp_path, monkeypatch):
    p = tmp_path / "server.toml"
    p.write_text('[server]\nport = 9000\n[moe]\ntop_k = 3\n[core.per_core]\nkv_cache_mb = 7\n[newsection]\nx = 1\n')
    monkeypatch.setenv("OPENMINI__SERVER__HOST", "127.0.0.1")
    cfg = ServerConfig.from_file(str(p))
    assert cfg.server.port == 9000 and cfg.server.host == "127.0.0.1"
    assert cfg.moe.top_k == 3 and cfg.moe.cycle_period == 3  # default kept
    assert cfg.core.per_core.kv_cache_mb == 7 and cfg.extra["newsection"] == {"x": 1}
    assert ServerConfig().validate() == []
    import pathlib
    shipped = pathlib.Path(__file__).resolve().parents[1] / "config" / "server.toml"
    load_config(str(shipped))


def test_gguf_roundtrip_and_tokenizer(tmp_path):
    from openmini_v1_b200.models.loader import load_gguf_model, save_gguf_model
    m = DecoderLM(tiny(), device="cpu", seed=4)
    T = 7
    i32 = dict(dtype=torch.int32)
    fb = lambda: ForwardBatch(torch.arange(50, 50 + T, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                              torch.arange(2, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                              torch.tensor([T - 1]))
    ref_logits = m.logits(m(fb(), m.allocate_kv(2)))
    for quant, tol in (("f32", 1e-5), ("q8_0", 5e-2)):
        path = str(tmp_path / f"m_{quant}.gguf")
        save_gguf_model(m, path, quant, tokenizer_tokens=["<unk>", "<s>", "</s>", "▁hi", "▁there"])
        m2 = load_gguf_model(path, device="cpu")
        out = m2.logits(m2(fb(), m2.allocate_kv(2)))
        assert (out - ref_logits).abs().max().item() < tol * max(1.0, ref_logits.abs().max().item()), quant
    from openmini_v1_b200.gguf.reader import GGUFReader
    tok = GGUFTokenizer.from_gguf(GGUFReader(path))
    ids = tok.encode("hi there")
    assert ids == [1, 3, 4] and tok.decode(ids) == "hi there"


def test_incremental_decoder_utf8():
    tok = ByteTokenizer()
    ids = tok.encode("héllo ✓", add_bos=False)
    d = IncrementalDecoder(tok)
    assert "".join(d.push(i) for i in ids) == "héllo ✓"


def test_health_middleware_errors_hardware(stack):
    from openmini_v1_b200.errors import KVCacheExhausted, OpenMiniError
    from openmini_v1_b200.hardware.detect import classify, detect_hardware, CpuInfo, GpuInfo
    from openmini_v1_b200.serve.middleware import mask_sensitive_data
    aeng, tok = stack[0], stack[1]
    c = TestClient(create_app(aeng, tok, "tiny"))
    assert c.get("/health/live").json() == {"status": "alive"}
    r = c.get("/health/ready")
    assert r.status_code in (200, 503) and {x["name"] for x in r.json()["components"]} >= {"gpu", "model"}
    r = c.get("/health", headers={"x-request-id": "abc"})
    assert r.headers["x-request-id"] == "abc"
    assert "***MASKED***" in mask_sensitive_data("Bearer eyJhbGciOiJIUzI1NiJ9 api_key=sk-123")
    assert "eyJ" not in mask_sensitive_data("Authorization: Bearer eyJhbGciOiJIUzI1NiJ9")
    e = KVCacheExhausted("no blocks", code=7, need=3)
    assert isinstance(e, OpenMiniError) and e.code == "ENG007" and e.http_status == 503
    assert e.to_dict()["need"] == 3
    hp = detect_hardware(nvml=None)
    assert hp.cpu.cores_logical >= 1 and hp.level in ("cpu_only", "gpu_other", "blackwell", "blackwell_nvswitch")
    g = [GpuInfo(i, "B200", (10, 0), 180 << 30, 148, 1965, 1000.0, 18) for i in range(8)]
    assert classify(CpuInfo("x86_64", 8, 4), g, 0)[0] == "blackwell_nvswitch"


class _FakeNVML:
    NVML_CLOCK_SM = 1

    class _Mem:
        total = 183359 << 20

    def nvmlInit(self): pass
    def nvmlShutdown(self): pass
    def nvmlDeviceGetCount(self): return 2
    def nvmlDeviceGetHandleByIndex(self, i): return i
    def nvmlDeviceGetName(self, h): return b"NVIDIA B200"
    def nvmlDeviceGetCudaComputeCapability(self, h): return (10, 0)
    def nvmlDeviceGetMemoryInfo(self, h): return self._Mem()
    def nvmlDeviceGetNumGpuCores(self, h): return 148 * 128
    def nvmlDeviceGetMaxClockInfo(self, h, t): return 1965
    def nvmlDeviceGetEnforcedPowerLimit(self, h): return 1000000
    def nvmlDeviceGetNvLinkState(self, h, l): return 1


def test_hardware_detection_fake_nvml():
    from openmini_v1_b200.hardware.detect import detect_hardware
    hp = detect_hardware(nvml=_FakeNVML())
    assert len(hp.gpus) == 2 and hp.gpus[0].sm_count == 148 and hp.gpus[0].nvlink_active == 18
    assert hp.level == "blackwell" and hp.strategy["tp"] == 2
