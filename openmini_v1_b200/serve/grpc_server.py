"""gRPC ``openmini.OpenMini`` service (grpcio, generic handlers, no codegen).

Behaviour of the reference's OpenMiniService
(openmini-server/src/service/grpc/server.rs:43-383,1114): Chat builds a prompt
from the session's stored memory plus the request messages ("role: content"
lines) and streams one ChatResponse per generated token, finishing with usage;
HealthCheck reports engine state. ImageUnderstanding(-Stream) run the vision
encoder and SpeechToText the audio encoder, then the engine, and TextToSpeech the
TTS model and vocoder, when the server was started with them (``vision``,
``speech``, ``tts``); otherwise they answer UNIMPLEMENTED instead of synthetic output.
Session memory is kept in SQLite (the reference's database), see ``SessionStore``.
"""
from __future__ import annotations

import asyncio
import os
import sqlite3
import threading
import time

import grpc

from ..engine.request import SamplingParams
from ..engine.tokenizer import IncrementalDecoder
from . import proto


class SessionStore:
    """SQLite message history per session (reference: S/db sessions/messages, WAL pool)."""

    def __init__(self, path: str = ":memory:", max_messages: int = 16):
        if path != ":memory:":
            os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        self.db = sqlite3.connect(path, check_same_thread=False)
        self.lock = threading.Lock()
        self.max_messages = max_messages
        with self.lock:
            if path != ":memory:":
                self.db.execute("PRAGMA journal_mode=WAL")
            self.db.execute("CREATE TABLE IF NOT EXISTS messages (session TEXT, ts REAL, role TEXT, content TEXT)")
            self.db.execute("CREATE INDEX IF NOT EXISTS idx_session ON messages(session, ts)")
            self.db.commit()

    def history(self, session: str) -> list:
        with self.lock:
            rows = self.db.execute("SELECT role, content FROM messages WHERE session=? ORDER BY ts DESC LIMIT ?",
                                   (session, self.max_messages)).fetchall()
        return [{"role": r, "content": c} for r, c in reversed(rows)]

    def add(self, session: str, role: str, content: str):
        with self.lock:
            self.db.execute("INSERT INTO messages VALUES (?, ?, ?, ?)", (session, time.time(), role, content))
            self.db.commit()


class OpenMiniServicer:
    def __init__(self, aengine, tokenizer, store: SessionStore | None = None, metrics=None, default_max_tokens=256,
                 vision=None, speech=None, tts=None):
        self.vision = vision
        self.tts = tts
        self.speech = speech
        self.aengine = aengine
        self.tok = tokenizer
        self.store = store or SessionStore()
        self.metrics = metrics
        self.default_max = default_max_tokens

    async def Chat(self, request_iterator, context):
        async for req in request_iterator:
            sid = req.session_id or f"session-{time.time_ns()}"
            msgs = self.store.history(sid) + [{"role": m.role, "content": m.content} for m in req.messages]
            prompt = "\n".join(f"{m['role']}: {m['content']}" for m in msgs) + "\nassistant:"
            ids = self.tok.encode(prompt)
            sp = SamplingParams(temperature=req.temperature if req.temperature > 0 else 0.0,
                                max_tokens=req.max_tokens if req.max_tokens > 0 else self.default_max, top_p=0.9)
            dec = IncrementalDecoder(self.tok)
            text, n = [], 0
            try:
                async for out in self.aengine.generate(ids, sp):
                    piece = dec.push(out.new_token_ids[0])
                    text.append(piece)
                    n += 1
                    if req.stream and not out.finished:
                        yield proto.ChatResponse(session_id=sid, token=piece, finished=False)
            except RuntimeError as e:
                await context.abort(grpc.StatusCode.INVALID_ARGUMENT, str(e))
            full = "".join(text)
            for m in req.messages:
                self.store.add(sid, m.role, m.content)
            self.store.add(sid, "assistant", full)
            usage = proto.UsageInfo(prompt_tokens=len(ids), completion_tokens=n, total_tokens=len(ids) + n)
            yield proto.ChatResponse(session_id=sid, token="" if req.stream else full, finished=True, usage=usage)

    async def HealthCheck(self, request, context):
        ok = self.aengine.alive and self.aengine.error is None
        return proto.HealthResponse(healthy=ok, message="ok" if ok else repr(self.aengine.error))

    async def ImageUnderstanding(self, request, context):
        if self.vision is None:
            await context.abort(grpc.StatusCode.UNIMPLEMENTED, "this server has no vision encoder loaded")
        try:
            text, _, _ = await self.vision.answer(request.image_data, request.question)
        except Exception as e:
            await context.abort(grpc.StatusCode.INVALID_ARGUMENT, f"image: {e}")
        return proto.ImageResponse(session_id=request.session_id, token=text, finished=True)

    async def ImageUnderstandingStream(self, request, context):
        if self.vision is None:
            await context.abort(grpc.StatusCode.UNIMPLEMENTED, "this server has no vision encoder loaded")
        try:
            async for piece, fin, _, _ in self.vision.stream(request.image_data, request.question):
                yield proto.ImageResponse(session_id=request.session_id, token=piece, finished=fin)
        except Exception as e:
            await context.abort(grpc.StatusCode.INVALID_ARGUMENT, f"image: {e}")

    async def SpeechToText(self, request_iterator, context):
        """Client-streamed audio chunks (one clip); the transcript is streamed back."""
        if self.speech is None:
            await context.abort(grpc.StatusCode.UNIMPLEMENTED, "this server has no audio encoder loaded")
        import math
        chunks, sid, lang = [], "", ""
        async for req in request_iterator:
            chunks.append(req.audio_data)
            sid, lang = req.session_id or sid, req.language or lang
        try:
            lps = []
            async for piece, fin, lp in self.speech.stream(b"".join(chunks), lang):
                lps.append(lp)
                conf = math.exp(sum(lps) / len(lps)) if lps else 0.0
                yield proto.SpeechToTextResponse(session_id=sid, text=piece, finished=fin, confidence=conf)
        except Exception as e:
            await context.abort(grpc.StatusCode.INVALID_ARGUMENT, f"audio: {e}")

    async def TextToSpeech(self, request, context):
        """One WAV clip streamed as byte chunks (header first); the last has finished=True."""
        if self.tts is None:
            await context.abort(grpc.StatusCode.UNIMPLEMENTED, "this server has no TTS model loaded")
        from ..models.tts import validate_request
        try:
            validate_request(request.text, request.speed or 1.0, request.pitch)
        except ValueError as e:
            await context.abort(grpc.StatusCode.INVALID_ARGUMENT, str(e))
        async for chunk, fin in self.tts.stream(request.text, request.voice, request.speed, request.pitch):
            yield proto.TextToSpeechResponse(session_id=request.session_id, audio_data=chunk, finished=fin)

    async def _unimplemented(self, request, context):
        await context.abort(grpc.StatusCode.UNIMPLEMENTED, "this server has no vision / speech encoder loaded")

    async def _unimplemented_stream(self, request, context):
        await context.abort(grpc.StatusCode.UNIMPLEMENTED, "this server has no vision / speech encoder loaded")
        yield  # pragma: no cover

    async def OmniChat(self, request_iterator, context):
        async for req in request_iterator:
            if req.WhichOneof("input") != "text":
                await context.abort(grpc.StatusCode.UNIMPLEMENTED, "only text input is served")
            ids = self.tok.encode(f"user: {req.text}\nassistant:")
            sp = SamplingParams(temperature=req.temperature if req.temperature > 0 else 0.0,
                                max_tokens=req.max_tokens if req.max_tokens > 0 else self.default_max)
            dec, n, text = IncrementalDecoder(self.tok), 0, []
            async for out in self.aengine.generate(ids, sp):
                piece = dec.push(out.new_token_ids[0])
                n += 1
                text.append(piece)
                if req.stream and not out.finished:
                    yield proto.OmniChatResponse(session_id=req.session_id, text=piece, finished=False)
            yield proto.OmniChatResponse(session_id=req.session_id, text="" if req.stream else "".join(text),
                                         finished=True,
                                         usage=proto.UsageInfo(prompt_tokens=len(ids), completion_tokens=n,
                                                               total_tokens=len(ids) + n))


def _handler(servicer):
    unary_unary, unary_stream, stream_stream = (grpc.unary_unary_rpc_method_handler,
                                                grpc.unary_stream_rpc_method_handler,
                                                grpc.stream_stream_rpc_method_handler)
    h = {}
    for name, (req, resp, cs, ss) in proto.METHODS.items():
        de = proto.message(req).FromString
        se = proto.message(resp).SerializeToString
        fn = getattr(servicer, name, None)
        if fn is None:
            fn = servicer._unimplemented_stream if ss else servicer._unimplemented
        if cs and ss:
            h[name] = stream_stream(fn, request_deserializer=de, response_serializer=se)
        elif ss:
            h[name] = unary_stream(fn, request_deserializer=de, response_serializer=se)
        else:
            h[name] = unary_unary(fn, request_deserializer=de, response_serializer=se)
    return grpc.method_handlers_generic_handler(proto.SERVICE, h)


async def start_grpc_server(servicer, addr: str = "127.0.0.1:50051", max_message_mb: int = 100):
    opts = [("grpc.max_send_message_length", max_message_mb << 20),
            ("grpc.max_receive_message_length", max_message_mb << 20)]
    server = grpc.aio.server(options=opts)
    server.add_generic_rpc_handlers((_handler(servicer),))
    port = server.add_insecure_port(addr)
    await server.start()
    return server, port


class OpenMiniClient:
    """Minimal async client (reference: openmini-client/client.py)."""

    def __init__(self, addr: str):
        self.channel = grpc.aio.insecure_channel(addr)

    def _call(self, name):
        req, resp, cs, ss = proto.METHODS[name]
        kind = ("stream_stream" if cs and ss else "unary_stream" if ss else "stream_unary" if cs
                else "unary_unary")
        return getattr(self.channel, kind)(f"/{proto.SERVICE}/{name}",
                                           request_serializer=proto.message(req).SerializeToString,
                                           response_deserializer=proto.message(resp).FromString)

    async def health(self) -> bool:
        r = await self._call("HealthCheck")(proto.HealthRequest())
        return r.healthy

    async def chat(self, messages, session_id="", max_tokens=16, temperature=0.0, stream=True):
        async def reqs():
            yield proto.ChatRequest(session_id=session_id, stream=stream, max_tokens=max_tokens,
                                    temperature=temperature,
                                    messages=[proto.Message(role=r, content=c) for r, c in messages])
        out = []
        async for r in self._call("Chat")(reqs()):
            out.append(r)
        return out

    async def close(self):
        await self.channel.close()
