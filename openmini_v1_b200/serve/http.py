"""HTTP API (FastAPI).

OpenAI-style surface: ``POST /v1/completions`` (prompt text or token ids,
optional SSE streaming), ``POST /v1/chat/completions``, ``GET /v1/models``,
``GET /health``, ``GET /metrics`` (Prometheus text).

Reference-compatible surface under ``/api/v1`` (routes of
openmini-server/src/service/http/server.rs:213-268): ``chat``,
``chat/stream`` (SSE), ``health``, ``models``, ``metrics``,
``inference/{compute,batch,stats,config,reset}``. The reference answers chat
with placeholder strings; here every chat route runs the engine. The image,
speech-to-text and text-to-speech routes run their models when the server loaded
them (/api/v1/image/understand, /api/v1/stt, /api/v1/tts) and answer 501 otherwise.
"""
from __future__ import annotations

import json
import math
import time
import uuid

from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from ..engine.request import SamplingParams
from ..engine.tokenizer import IncrementalDecoder
from .metrics import Metrics


def _params(body: dict, default_max: int = 16) -> SamplingParams:
    return SamplingParams(
        temperature=float(body.get("temperature", 1.0)), top_p=float(body.get("top_p", 1.0)),
        top_k=int(body.get("top_k", 0) or 0), repetition_penalty=float(body.get("repetition_penalty", 1.0)),
        max_tokens=int(body["max_tokens"]) if body.get("max_tokens") is not None else default_max,
        min_tokens=int(body.get("min_tokens", 0)), stop_token_ids=list(body.get("stop_token_ids", []) or []),
        ignore_eos=bool(body.get("ignore_eos", False)), seed=body.get("seed"),
        logprobs=bool(body.get("logprobs", False)))


def chat_prompt(messages) -> str:
    """Messages -> prompt, one "role: content" line per message (the reference's format)."""
    lines = [f"{m.get('role', 'user')}: {m.get('content', '')}" for m in messages]
    return "\n".join(lines) + "\nassistant:"


def create_app(aengine, tokenizer, model_name: str = "openmini", metrics: Metrics | None = None,
               config=None, trainer_factory=None, vision=None, speech=None, tts=None) -> FastAPI:
    app = FastAPI(title="openmini_v1_b200")

    async def _bad_request(request, exc):
        # a request body with fields of the wrong type or shape (for example max_tokens: [])
        # fails while being read into engine parameters: that is the client's error
        return JSONResponse({"error": f"bad request: {type(exc).__name__}: {exc}"}, status_code=400)

    for exc_type in (TypeError, ValueError, KeyError, AttributeError, IndexError):
        app.add_exception_handler(exc_type, _bad_request)
    metrics = metrics or Metrics()
    metrics.model_loaded.set(1)
    started = time.time()
    app.state.metrics = metrics
    app.state.engine = aengine

    def to_ids(prompt):
        if isinstance(prompt, str):
            return tokenizer.encode(prompt)
        if isinstance(prompt, list) and all(isinstance(t, int) for t in prompt):
            return prompt
        raise HTTPException(400, "prompt must be a string or a list of token ids")

    async def run_one(ids, sp, endpoint):
        t0 = time.time()
        metrics.active_requests.inc()
        toks, lps, reason, first = [], [], None, None
        try:
            async for out in aengine.generate(ids, sp):
                if first is None:
                    first = time.time()
                    metrics.ttft_ms.observe((first - t0) * 1e3)
                toks = list(out.output_token_ids)
                reason = out.finish_reason
                if out.logprobs:
                    lps = out.logprobs
        except RuntimeError as e:
            metrics.observe_request(endpoint, "error", time.time() - t0)
            raise HTTPException(400, str(e))
        finally:
            metrics.active_requests.dec()
        dt = time.time() - t0
        metrics.observe_request(endpoint, "ok", dt)
        metrics.observe_tokens(len(toks))
        metrics.observe_tokens(len(ids), "prompt")
        if first is not None and len(toks) > 1:
            metrics.tpot_ms.observe((time.time() - first) * 1e3 / (len(toks) - 1))
        return toks, lps, reason

    def sse(gen_fn):
        async def body():
            async for chunk in gen_fn():
                yield f"data: {json.dumps(chunk)}\n\n"
            yield "data: [DONE]\n\n"
        return StreamingResponse(body(), media_type="text/event-stream")

    # ---------------------------------------------------------------- OpenAI-style
    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        prompt = body.get("prompt", "")
        ids = to_ids(prompt)
        try:
            sp = _params(body)
            sp.validate()
        except ValueError as e:
            raise HTTPException(400, str(e))
        cid = f"cmpl-{uuid.uuid4().hex[:16]}"
        created = int(time.time())
        if body.get("stream"):
            async def gen():
                dec = IncrementalDecoder(tokenizer)
                t0 = time.time()
                metrics.active_requests.inc()
                n = 0
                try:
                    async for out in aengine.generate(ids, sp):
                        n += 1
                        tid = out.new_token_ids[0]
                        yield {"id": cid, "object": "text_completion", "created": created, "model": model_name,
                               "choices": [{"index": 0, "text": dec.push(tid), "token_ids": [tid],
                                            "finish_reason": out.finish_reason}]}
                finally:
                    metrics.active_requests.dec()
                    metrics.observe_request("/v1/completions", "ok", time.time() - t0)
                    metrics.observe_tokens(n)
            return sse(gen)
        toks, lps, reason = await run_one(ids, sp, "/v1/completions")
        choice = {"index": 0, "text": tokenizer.decode(toks), "token_ids": toks, "finish_reason": reason}
        if sp.logprobs:
            choice["logprobs"] = {"token_logprobs": lps}
        return {"id": cid, "object": "text_completion", "created": created, "model": model_name,
                "choices": [choice],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(toks),
                          "total_tokens": len(ids) + len(toks)}}

    @app.post("/v1/chat/completions")
    async def chat_completions(req: Request):
        body = await req.json()
        ids = tokenizer.encode(chat_prompt(body.get("messages", [])))
        sp = _params(body)
        toks, _, reason = await run_one(ids, sp, "/v1/chat/completions")
        return {"id": f"chatcmpl-{uuid.uuid4().hex[:16]}", "object": "chat.completion", "created": int(time.time()),
                "model": model_name,
                "choices": [{"index": 0, "message": {"role": "assistant", "content": tokenizer.decode(toks)},
                             "finish_reason": reason}],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(toks),
                          "total_tokens": len(ids) + len(toks)}}

    def _models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "openmini"}]}

    def _health():
        ok = aengine.alive and aengine.error is None
        return {"status": "healthy" if ok else "unhealthy", "version": "0.1.0",
                "uptime": int(time.time() - started), "model": model_name,
                "error": None if aengine.error is None else repr(aengine.error)}

    @app.get("/v1/models")
    async def models():
        return _models()

    @app.get("/health")
    async def health():
        h = _health()
        return JSONResponse(h, status_code=200 if h["status"] == "healthy" else 503)

    @app.get("/metrics")
    async def prom():
        metrics.update_engine(aengine.engine)
        return PlainTextResponse(metrics.render().decode(), media_type="text/plain; version=0.0.4")

    # ---------------------------------------------------------------- /api/v1 (reference routes)
    @app.get("/api/v1/health")
    async def api_health():
        return _health()

    @app.get("/api/v1/models")
    async def api_models():
        return _models()

    @app.get("/api/v1/metrics")
    async def api_metrics():
        metrics.update_engine(aengine.engine)
        return PlainTextResponse(metrics.render().decode())

    @app.post("/api/v1/chat")
    async def api_chat(req: Request):
        body = await req.json()
        msgs = body.get("messages") or [{"role": "user", "content": body.get("message", "")}]
        ids = tokenizer.encode(chat_prompt(msgs))
        toks, _, reason = await run_one(ids, _params(body, 64), "/api/v1/chat")
        return {"session_id": body.get("session_id", str(uuid.uuid4())), "response": tokenizer.decode(toks),
                "finish_reason": reason, "usage": {"prompt_tokens": len(ids), "completion_tokens": len(toks)}}

    @app.post("/api/v1/chat/stream")
    async def api_chat_stream(req: Request):
        body = await req.json()
        msgs = body.get("messages") or [{"role": "user", "content": body.get("message", "")}]
        ids = tokenizer.encode(chat_prompt(msgs))
        sp = _params(body, 64)
        sid = body.get("session_id", str(uuid.uuid4()))

        async def gen():
            dec = IncrementalDecoder(tokenizer)
            async for out in aengine.generate(ids, sp):
                yield {"session_id": sid, "token": dec.push(out.new_token_ids[0]), "finished": out.finished}
        return sse(gen)

    from ..models.hp_pipeline import HighPerformancePipeline
    pipeline = HighPerformancePipeline()

    @app.post("/api/v1/inference/compute")
    async def api_compute(req: Request):
        """Raw attention over client-supplied q, k, v ([seq, dim] lists, or [seq, heads, head_dim])
        through the high-performance pipeline on the engine's device (strategy chosen by length)."""
        import torch
        body = await req.json()
        try:
            q, k, v = (torch.tensor(body[n], dtype=torch.float32) for n in ("q", "k", "v"))
        except Exception:
            raise HTTPException(400, "q, k, v must be numeric arrays")
        if q.dim() == 2:
            q, k, v = q[:, None], k[:, None], v[:, None]
        if q.dim() != 3 or k.shape != v.shape or q.shape[2] != k.shape[2] or q.shape[1] % k.shape[1]:
            raise HTTPException(400, "shape mismatch")
        dev = getattr(getattr(aengine, "engine", None), "device", torch.device("cpu"))
        causal = bool(body.get("causal", False)) and q.shape[0] <= k.shape[0]
        t0 = time.time()
        o, strat = pipeline.forward(q.to(dev), k.to(dev), v.to(dev), causal=causal)
        o = o.cpu()
        if o.shape[1] == 1 and len(body["q"]) and not isinstance(body["q"][0][0], list):
            o = o[:, 0]
        return {"output": o.tolist(), "strategy": strat, "inference_time_ms": (time.time() - t0) * 1e3,
                "stats": {"calls": pipeline.stats.calls, "by_strategy": dict(pipeline.stats.by_strategy)}}

    @app.post("/api/v1/inference/batch")
    async def api_batch(req: Request):
        body = await req.json()
        prompts = body.get("prompts", [])
        sp = _params(body)
        import asyncio
        res = await asyncio.gather(*[run_one(to_ids(p), sp, "/api/v1/inference/batch") for p in prompts])
        return {"results": [{"token_ids": t, "text": tokenizer.decode(t), "finish_reason": r} for t, _, r in res]}

    @app.get("/api/v1/inference/stats")
    async def api_stats():
        e = aengine.engine
        return {"engine": dict(e.stats), "kv_blocks_free": e.bm.num_free(), "kv_blocks_total": e.bm.num_blocks,
                "prefix_hit_rate": e.bm.prefix_hit_rate(), "waiting": len(e.sched.waiting),
                "running": len(e.sched.running)}

    @app.get("/api/v1/inference/config")
    async def api_config():
        import dataclasses
        return {"engine": dataclasses.asdict(aengine.engine.cfg), "model": aengine.engine.model.cfg.to_dict()}

    @app.post("/api/v1/inference/reset")
    async def api_reset():
        e = aengine.engine
        e.bm.reset_prefix_cache()
        for k in e.stats:
            e.stats[k] = 0
        return {"status": "ok"}

    @app.post("/api/v1/image/understand")
    async def image_understand(body: dict):
        """{"image": base64 bytes, "question": str, "max_tokens"?: int, "temperature"?: float}"""
        if vision is None:
            return JSONResponse({"error": "/api/v1/image/understand needs a vision encoder, which is not loaded"},
                                status_code=501)
        import base64
        try:
            data = base64.b64decode(body["image"])
            text, pt, n = await vision.answer(data, str(body.get("question", "Describe the image.")),
                                              int(body.get("max_tokens", 0)), float(body.get("temperature", 0.0)))
        except (KeyError, ValueError, OSError) as e:
            return JSONResponse({"error": f"bad image request: {e}"}, status_code=400)
        return {"answer": text, "usage": {"prompt_tokens": pt, "completion_tokens": n, "total_tokens": pt + n}}

    @app.post("/api/v1/stt")
    async def stt(body: dict):
        """{"audio": base64 WAV or .npy bytes, "language"?: str, "max_tokens"?: int}"""
        if speech is None:
            return JSONResponse({"error": "/api/v1/stt needs an audio encoder, which is not loaded"}, status_code=501)
        import base64
        try:
            data = base64.b64decode(body["audio"])
            text = []
            async for piece, fin, lp in speech.stream(data, str(body.get("language", "")),
                                                      int(body.get("max_tokens", 0))):
                text.append(piece)
        except (KeyError, ValueError, OSError, EOFError) as e:
            return JSONResponse({"error": f"bad audio request: {e}"}, status_code=400)
        return {"text": "".join(text), "tokens": len(text)}

    @app.post("/api/v1/tts")
    async def tts_route(body: dict):
        """{"text": str, "voice"?: str, "language"?: str, "speed"?: 0.25-4, "pitch"?: -20-20}
        -> {"audio_data": base64 WAV, "sample_rate", "duration_s"}"""
        if tts is None:
            return JSONResponse({"error": "/api/v1/tts needs a TTS model, which is not loaded"}, status_code=501)
        import base64
        from ..models.tts import validate_request
        try:
            text, speed, pitch = str(body["text"]), float(body.get("speed", 1.0)), float(body.get("pitch", 0.0))
            validate_request(text, speed, pitch)
        except (KeyError, ValueError, TypeError) as e:
            return JSONResponse({"error": f"bad tts request: {e}"}, status_code=400)
        wav = await tts.synthesize(text, str(body.get("voice", "default")), speed, pitch)
        sr = tts.model.cfg.sample_rate
        return {"audio_data": base64.b64encode(wav).decode(), "sample_rate": sr,
                "duration_s": (len(wav) - 44) / 2 / sr}

    from .training_api import mount_training
    mount_training(app, trainer_factory)
    from .health import HealthChecker, mount_health
    mount_health(app, HealthChecker(aengine))
    from .middleware import apply_middlewares
    apply_middlewares(app)
    return app
