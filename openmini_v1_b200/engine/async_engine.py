"""Asynchronous front of the engine for servers.

One background thread owns the ``LLMEngine`` and runs ``step()`` while work
is pending; requests are submitted from any thread / event loop and their
outputs are streamed back through per-request queues. This replaces the
reference's AsyncInferencePool + TaskScheduler pairing
(openmini-server/src/service/worker/async_pool.rs:13-181,
openmini-server/src/service/scheduler/mod.rs:375-630), whose engine closure
was a placeholder, with continuous batching across all in-flight requests.
"""
from __future__ import annotations

import asyncio
import itertools
import queue
import threading
import time

from .request import SamplingParams


class AsyncLLMEngine:
    def __init__(self, engine, idle_sleep_s: float = 0.001):
        self.engine = engine
        self._inbox: queue.Queue = queue.Queue()
        self._subs: dict = {}
        self._ids = itertools.count()
        self._stop = threading.Event()
        self._idle = idle_sleep_s
        self.error: BaseException | None = None
        self.started_at = time.time()
        self._thread = threading.Thread(target=self._loop, name="openmini-engine", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------ engine thread
    def _loop(self):
        eng = self.engine
        while not self._stop.is_set():
            try:
                while True:
                    kind, payload = self._inbox.get_nowait()
                    if kind == "add":
                        rid, toks, params, sink, prio, img = payload
                        try:
                            eng.add_request(rid, toks, params, priority=prio, image_embeds=img)
                            self._subs[rid] = sink
                        except Exception as e:  # invalid request: report to its caller only
                            sink(("error", str(e)))
                    elif kind == "abort":
                        eng.abort_request(payload)
                        sink = self._subs.pop(payload, None)
                        if sink:
                            sink(("aborted", None))
            except queue.Empty:
                pass
            if not eng.has_unfinished():
                time.sleep(self._idle)
                continue
            try:
                outs = eng.step()
            except BaseException as e:  # engine failure: fail every waiter, keep serving
                self.error = e
                for rid, sink in list(self._subs.items()):
                    sink(("error", repr(e)))
                    eng.abort_request(rid)
                self._subs.clear()
                continue
            for o in outs:
                sink = self._subs.get(o.request_id)
                if sink is None:
                    continue
                sink(("output", o))
                if o.finished:
                    self._subs.pop(o.request_id, None)

    def shutdown(self):
        self._stop.set()
        self._thread.join(timeout=10)

    @property
    def alive(self) -> bool:
        return self._thread.is_alive()

    # ------------------------------------------------------------ client side
    def submit(self, prompt_token_ids, params: SamplingParams, sink, request_id: str | None = None,
               priority: int = 0, image_embeds: tuple | None = None) -> str:
        rid = request_id or f"req-{next(self._ids)}"
        params.validate()
        self._inbox.put(("add", (rid, list(prompt_token_ids), params, sink, priority, image_embeds)))
        return rid

    def abort(self, request_id: str):
        self._inbox.put(("abort", request_id))

    async def generate(self, prompt_token_ids, params: SamplingParams, request_id: str | None = None,
                       priority: int = 0, image_embeds: tuple | None = None):
        """Async iterator of RequestOutput (one per generated token)."""
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()

        def sink(item):
            loop.call_soon_threadsafe(q.put_nowait, item)

        rid = self.submit(prompt_token_ids, params, sink, request_id, priority, image_embeds)
        try:
            while True:
                kind, val = await q.get()
                if kind == "error":
                    raise RuntimeError(val)
                if kind == "aborted":
                    return
                yield val
                if val.finished:
                    return
        except (asyncio.CancelledError, GeneratorExit):
            self.abort(rid)
            raise

    def generate_sync(self, prompt_token_ids, params: SamplingParams, timeout: float = 600.0):
        """Blocking helper: returns the final RequestOutput."""
        q: queue.Queue = queue.Queue()
        self.submit(prompt_token_ids, params, q.put)
        deadline = time.time() + timeout
        last = None
        while True:
            kind, val = q.get(timeout=max(0.0, deadline - time.time()))
            if kind == "error":
                raise RuntimeError(val)
            if kind == "aborted":
                return last
            last = val
            if val.finished:
                return val
