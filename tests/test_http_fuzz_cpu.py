"""HTTP robustness (hypothesis): random JSON bodies -- wrong types, missing or
extra fields, out-of-range numbers -- sent to every POST route of the inference API
get a client error or a success, never a server error, and the engine keeps
serving afterwards."""
import pytest
from fastapi.testclient import TestClient
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from openmini_v1_b200.engine.async_engine import AsyncLLMEngine
from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.tokenizer import ByteTokenizer
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM
from openmini_v1_b200.serve.http import create_app

ROUTES = ["/v1/completions", "/v1/chat/completions", "/api/v1/chat", "/api/v1/chat/stream",
          "/api/v1/inference/compute", "/api/v1/inference/batch", "/api/v1/image/understand", "/api/v1/stt",
          "/api/v1/tts"]
KEYS = ["prompt", "messages", "max_tokens", "temperature", "top_p", "top_k", "stream", "seed", "stop", "n",
        "q", "k", "v", "seq_len", "inputs", "text", "speed", "image", "audio", "question", "role", "content"]
leaf = st.one_of(st.none(), st.booleans(), st.integers(-10 ** 6, 10 ** 6), st.floats(allow_nan=False, allow_infinity=False, width=32),
                 st.text(max_size=12))
value = st.recursive(leaf, lambda ch: st.one_of(st.lists(ch, max_size=4),
                                                st.dictionaries(st.sampled_from(KEYS), ch, max_size=3)),
                     max_leaves=8)
bodies = st.dictionaries(st.sampled_from(KEYS), value, max_size=5)


@pytest.fixture(scope="module")
def client():
    eng = LLMEngine(DecoderLM(tiny(), device="cpu", seed=1),
                    EngineConfig(max_num_seqs=4, max_model_len=128, use_cuda_graph=False))
    aeng = AsyncLLMEngine(eng)
    with TestClient(create_app(aeng, ByteTokenizer(), "tiny"), raise_server_exceptions=False) as c:
        yield c
    aeng.shutdown()


@settings(max_examples=150, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(route=st.sampled_from(ROUTES), body=bodies)
def test_no_server_errors(client, route, body):
    if isinstance(body.get("max_tokens"), int):
        body["max_tokens"] = max(-5, min(body["max_tokens"], 8))   # keep each generation short
    r = client.post(route, json=body)
    assert r.status_code < 500 or r.status_code == 501, (route, body, r.status_code, r.text[:300])


def test_still_serving_after_fuzz(client):
    r = client.post("/v1/completions", json={"prompt": "hello", "max_tokens": 3, "temperature": 0.0})
    assert r.status_code == 200 and r.json()["usage"]["completion_tokens"] == 3
