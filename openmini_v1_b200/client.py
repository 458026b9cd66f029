"""Synchronous gRPC client of the ``openmini.OpenMini`` service.

Same surface as the reference's Python client (openmini-client/client.py:151-470):
a pool of channels used round-robin, per-call deadlines, retries with
exponential backoff on transient status codes (UNAVAILABLE, DEADLINE_EXCEEDED,
RESOURCE_EXHAUSTED), and the calls ``chat`` (streamed tokens or the whole
answer), ``chat_stream`` (iterator of tokens), ``image_understanding`` and
``health_check``. Messages are the protobuf classes of ``serve.proto``, so no
generated stubs are needed.

    with OpenMiniClient("127.0.0.1:50051", pool_size=2) as c:
        print(c.chat([("user", "hello")], max_tokens=16).text)
"""
from __future__ import annotations

import itertools
import threading
import time
from dataclasses import dataclass, field

import grpc

from .serve import proto

RETRYABLE = (grpc.StatusCode.UNAVAILABLE, grpc.StatusCode.DEADLINE_EXCEEDED, grpc.StatusCode.RESOURCE_EXHAUSTED)


@dataclass
class ChatResult:
    session_id: str
    text: str
    tokens: list = field(default_factory=list)
    prompt_tokens: int = 0
    completion_tokens: int = 0
    latency_s: float = 0.0
    ttft_s: float | None = None


class OpenMiniClient:
    def __init__(self, addr: str, pool_size: int = 1, timeout_s: float = 60.0, max_retries: int = 3,
                 backoff_s: float = 0.1, max_message_mb: int = 100):
        opts = [("grpc.max_send_message_length", max_message_mb << 20),
                ("grpc.max_receive_message_length", max_message_mb << 20)]
        self.addr = addr
        self.channels = [grpc.insecure_channel(addr, options=opts) for _ in range(max(1, pool_size))]
        self._rr = itertools.cycle(range(len(self.channels)))
        self._lock = threading.Lock()
        self.timeout_s = timeout_s
        self.max_retries = max_retries
        self.backoff_s = backoff_s
        self.stats = {"calls": 0, "retries": 0, "errors": 0}

    # ------------------------------------------------------------------ plumbing
    def _channel(self):
        with self._lock:
            return self.channels[next(self._rr)]

    def _stub(self, name, channel=None):
        req, resp, cs, ss = proto.METHODS[name]
        kind = ("stream_stream" if cs and ss else "unary_stream" if ss else "stream_unary" if cs
                else "unary_unary")
        return getattr(channel or self._channel(), kind)(
            f"/{proto.SERVICE}/{name}", request_serializer=proto.message(req).SerializeToString,
            response_deserializer=proto.message(resp).FromString)

    def _retry(self, fn):
        delay = self.backoff_s
        for attempt in range(self.max_retries + 1):
            self.stats["calls"] += 1
            try:
                return fn()
            except grpc.RpcError as e:
                if e.code() not in RETRYABLE or attempt == self.max_retries:
                    self.stats["errors"] += 1
                    raise
                self.stats["retries"] += 1
                time.sleep(delay)
                delay *= 2

    # ------------------------------------------------------------------ API
    def health_check(self) -> bool:
        try:
            return bool(self._retry(lambda: self._stub("HealthCheck")(proto.HealthRequest(),
                                                                         timeout=self.timeout_s)).healthy)
        except grpc.RpcError:
            return False

    def chat_stream(self, messages, session_id: str = "", max_tokens: int = 256, temperature: float = 0.0):
        """Yields ``ChatResponse`` messages (one per token, the last with ``finished`` and usage)."""
        req = proto.ChatRequest(session_id=session_id, stream=True, max_tokens=max_tokens, temperature=temperature,
                                messages=[proto.Message(role=r, content=c) for r, c in messages])
        yield from self._stub("Chat")(iter([req]), timeout=self.timeout_s)

    def chat(self, messages, session_id: str = "", max_tokens: int = 256, temperature: float = 0.0,
             stream: bool = True) -> ChatResult:
        def run():
            t0 = time.perf_counter()
            res = ChatResult(session_id=session_id, text="")
            req = proto.ChatRequest(session_id=session_id, stream=stream, max_tokens=max_tokens,
                                    temperature=temperature,
                                    messages=[proto.Message(role=r, content=c) for r, c in messages])
            pieces = []
            for r in self._stub("Chat")(iter([req]), timeout=self.timeout_s):
                if res.ttft_s is None:
                    res.ttft_s = time.perf_counter() - t0
                res.session_id = r.session_id
                if r.finished:
                    if r.token:
                        pieces.append(r.token)
                    res.prompt_tokens = r.usage.prompt_tokens
                    res.completion_tokens = r.usage.completion_tokens
                else:
                    pieces.append(r.token)
                    res.tokens.append(r.token)
            res.text = "".join(pieces)
            res.latency_s = time.perf_counter() - t0
            return res
        return self._retry(run)

    def image_understanding(self, image: bytes, question: str, session_id: str = "") -> str:
        r = self._retry(lambda: self._stub("ImageUnderstanding")(
            proto.ImageRequest(session_id=session_id, image_data=image, question=question), timeout=self.timeout_s))
        return r.token

    def close(self):
        for ch in self.channels:
            ch.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
