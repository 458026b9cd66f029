"""Host-side concurrency of the serving stack: a prioritised thread pool with
compute / IO / mixed presets, range partitioners (static, dynamic, guided), one
actor thread per CPU core with a router in front of them, and a bounded
connection pool.

GPU work is not parallelised here (one engine owns the device and batches every
request); these pieces carry the host work around it: tokenisation, detokenisation,
request parsing, client connections and CPU-side pre/post-processing.

Reference counterparts:
  ThreadPool, PoolConfig presets ........ openmini-server/src/service/thread/pool.rs:24-330
  TaskPartitioner, Dynamic/GuidedScheduler openmini-server/src/service/thread/strategy.rs:16-350
  PerCoreActor .......................... openmini-server/src/service/core_actor.rs:18-197
  CoreRouter (round robin, least connections, consistent hash)
                                          openmini-server/src/service/router.rs:14-185
  ConnectionPool ........................ openmini-server/src/service/server/connection.rs
The reference's per-core actor answers a fixed placeholder string; here an actor
runs the handler it is given (for example a call into the async engine).
"""
from __future__ import annotations

import bisect
import hashlib
import heapq
import itertools
import os
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable


# ----------------------------------------------------------------------------- thread pool

@dataclass
class PoolConfig:
    size: int = 0                  # 0: derived from the CPU count and the workload kind
    kind: str = "mixed"            # "compute" | "io" | "mixed"
    max_queue: int = 0             # 0: unbounded; otherwise execute() blocks when full
    name: str = "om-pool"

    def resolved_size(self) -> int:
        if self.size > 0:
            return self.size
        n = os.cpu_count() or 4
        return {"compute": n, "io": 4 * n, "mixed": 2 * n}.get(self.kind, n)

    @classmethod
    def compute_intensive(cls):
        return cls(kind="compute")

    @classmethod
    def io_intensive(cls):
        return cls(kind="io")

    @classmethod
    def mixed(cls):
        return cls(kind="mixed")


class ThreadPool:
    """Fixed set of worker threads over one priority queue (lower value first, FIFO
    within a priority). ``execute`` returns a future-like handle."""

    HIGH, NORMAL = 0, 10

    class Handle:
        def __init__(self):
            self._ev = threading.Event()
            self._res = None
            self._exc = None

        def result(self, timeout: float | None = None):
            if not self._ev.wait(timeout):
                raise TimeoutError("task not finished")
            if self._exc is not None:
                raise self._exc
            return self._res

        def done(self) -> bool:
            return self._ev.is_set()

    def __init__(self, config: PoolConfig | int | None = None):
        if isinstance(config, int):
            config = PoolConfig(size=config)
        self.config = config or PoolConfig()
        self._cv = threading.Condition()
        self._heap: list = []
        self._seq = itertools.count()
        self._active = 0
        self._pending = 0
        self._closed = False
        self._threads = [threading.Thread(target=self._worker, name=f"{self.config.name}-{i}", daemon=True)
                         for i in range(self.config.resolved_size())]
        for t in self._threads:
            t.start()

    @property
    def size(self) -> int:
        return len(self._threads)

    @property
    def active_count(self) -> int:
        return self._active

    def execute(self, fn: Callable, *args, priority: int = NORMAL, **kw) -> "ThreadPool.Handle":
        h = ThreadPool.Handle()
        with self._cv:
            if self._closed:
                raise RuntimeError("thread pool is shut down")
            while self.config.max_queue and len(self._heap) >= self.config.max_queue:
                self._cv.wait()
            heapq.heappush(self._heap, (priority, next(self._seq), fn, args, kw, h))
            self._pending += 1
            self._cv.notify_all()
        return h

    def execute_high_priority(self, fn: Callable, *args, **kw):
        return self.execute(fn, *args, priority=ThreadPool.HIGH, **kw)

    def map(self, fn: Callable, items) -> list:
        return [h.result() for h in [self.execute(fn, x) for x in items]]

    def _worker(self):
        while True:
            with self._cv:
                while not self._heap and not self._closed:
                    self._cv.wait()
                if not self._heap:
                    return
                _, _, fn, args, kw, h = heapq.heappop(self._heap)
                self._active += 1
                self._cv.notify_all()
            try:
                h._res = fn(*args, **kw)
            except BaseException as e:  # delivered to the caller through the handle
                h._exc = e
            finally:
                h._ev.set()
                with self._cv:
                    self._active -= 1
                    self._pending -= 1
                    self._cv.notify_all()

    def wait_completion(self, timeout: float | None = None) -> bool:
        end = None if timeout is None else time.monotonic() + timeout
        with self._cv:
            while self._pending:
                left = None if end is None else end - time.monotonic()
                if left is not None and left <= 0:
                    return False
                self._cv.wait(left)
        return True

    def shutdown(self, wait: bool = True):
        with self._cv:
            self._closed = True
            self._cv.notify_all()
        if wait:
            for t in self._threads:
                t.join()


def create_compute_pool() -> ThreadPool:
    return ThreadPool(PoolConfig.compute_intensive())


def create_io_pool() -> ThreadPool:
    return ThreadPool(PoolConfig.io_intensive())


# ----------------------------------------------------------------------------- partitioners

@dataclass
class TaskPartitioner:
    """Splits [0, total) into contiguous chunks for ``workers`` threads, never smaller
    than ``min_chunk`` (below that the per-task overhead dominates)."""
    workers: int = field(default_factory=lambda: os.cpu_count() or 4)
    min_chunk: int = 1024

    def optimal_parallelism(self, total: int) -> int:
        return max(1, min(self.workers, total // max(self.min_chunk, 1)))

    def partition_range(self, total: int) -> list[tuple[int, int]]:
        n = self.optimal_parallelism(total)
        base, extra = divmod(total, n)
        out, s = [], 0
        for i in range(n):
            e = s + base + (1 if i < extra else 0)
            if e > s:
                out.append((s, e))
            s = e
        return out

    def partition_to_cores(self, total: int) -> list[tuple[int, int, int]]:
        """(core id, start, end) with cores taken from this process's affinity mask."""
        try:
            cores = sorted(os.sched_getaffinity(0))
        except (AttributeError, OSError):
            cores = list(range(os.cpu_count() or 1))
        return [(cores[i % len(cores)], s, e) for i, (s, e) in enumerate(self.partition_range(total))]


class DynamicScheduler:
    """Fixed-size chunks handed out on demand (work stealing from one counter)."""

    def __init__(self, total: int, chunk: int):
        self.total, self.chunk = total, max(1, chunk)
        self._next = 0
        self._lock = threading.Lock()

    def next_chunk(self):
        with self._lock:
            if self._next >= self.total:
                return None
            s = self._next
            self._next = min(self.total, s + self.chunk)
            return s, self._next

    def remaining(self) -> int:
        return max(0, self.total - self._next)

    def reset(self):
        with self._lock:
            self._next = 0


class GuidedScheduler(DynamicScheduler):
    """Chunks of remaining / workers, shrinking towards ``min_chunk`` (OpenMP guided)."""

    def __init__(self, total: int, workers: int, min_chunk: int = 1):
        super().__init__(total, min_chunk)
        self.workers = max(1, workers)

    def next_chunk(self):
        with self._lock:
            rem = self.total - self._next
            if rem <= 0:
                return None
            n = max(self.chunk, -(-rem // self.workers))
            s = self._next
            self._next = min(self.total, s + n)
            return s, self._next


# ----------------------------------------------------------------------------- per-core actors + router

@dataclass
class CoreRequest:
    payload: Any
    session_id: str
    reply: "queue.Queue"


@dataclass
class CoreResponse:
    session_id: str
    ok: bool
    result: Any = None
    error: str | None = None


class PerCoreActor:
    """One thread pinned to one CPU core (where the OS allows it) serving requests from
    its own queue with ``handler(payload) -> result``."""

    def __init__(self, core_id: int, handler: Callable[[Any], Any], pin: bool = True):
        self.core_id = core_id
        self.handler = handler
        self.inbox: queue.Queue = queue.Queue()
        self.active_connections = 0
        self.served = 0
        self.pinned = False
        self._pin = pin
        self._thread = threading.Thread(target=self._run, name=f"core-{core_id}", daemon=True)
        self._thread.start()

    def _run(self):
        if self._pin and hasattr(os, "sched_setaffinity"):
            try:
                os.sched_setaffinity(threading.get_native_id(), {self.core_id})
                self.pinned = True
            except OSError:
                self.pinned = False
        while True:
            req = self.inbox.get()
            if req is None:
                return
            self.active_connections += 1
            try:
                resp = CoreResponse(req.session_id, True, self.handler(req.payload))
            except Exception as e:
                resp = CoreResponse(req.session_id, False, error=repr(e))
            self.active_connections -= 1
            self.served += 1
            req.reply.put(resp)

    def load(self) -> int:
        return self.active_connections + self.inbox.qsize()

    def stop(self):
        self.inbox.put(None)
        self._thread.join(5)


class CoreRouter:
    """Dispatches requests to per-core actors: ``round_robin``, ``least_connections``
    or ``consistent_hash`` (a ring of ``virtual_nodes`` points per actor, so a session
    keeps its actor and only 1/N of the sessions move when an actor is added)."""

    def __init__(self, actors: list[PerCoreActor], strategy: str = "round_robin", virtual_nodes: int = 64):
        if not actors:
            raise ValueError("at least one actor")
        self.actors = list(actors)
        self.strategy = strategy
        self._rr = itertools.count()
        self._ring: list[tuple[int, int]] = []
        for i, a in enumerate(self.actors):
            for v in range(virtual_nodes):
                self._ring.append((self._h(f"actor-{i}-core-{a.core_id}#{v}"), i))
        self._ring.sort()
        self._keys = [k for k, _ in self._ring]

    @staticmethod
    def _h(s: str) -> int:
        return int.from_bytes(hashlib.blake2b(s.encode(), digest_size=8).digest(), "little")

    def select(self, session_id: str) -> int:
        if self.strategy == "least_connections":
            return min(range(len(self.actors)), key=lambda i: self.actors[i].load())
        if self.strategy == "consistent_hash":
            i = bisect.bisect(self._keys, self._h(session_id)) % len(self._ring)
            return self._ring[i][1]
        return next(self._rr) % len(self.actors)

    def dispatch(self, payload, session_id: str = "") -> "queue.Queue":
        reply: queue.Queue = queue.Queue(maxsize=1)
        self.actors[self.select(session_id)].inbox.put(CoreRequest(payload, session_id, reply))
        return reply

    def call(self, payload, session_id: str = "", timeout: float | None = 30.0) -> CoreResponse:
        return self.dispatch(payload, session_id).get(timeout=timeout)

    def stop(self):
        for a in self.actors:
            a.stop()


def spawn_core_actors(handler: Callable, cores: list[int] | None = None, pin: bool = True) -> list[PerCoreActor]:
    if cores is None:
        try:
            cores = sorted(os.sched_getaffinity(0))
        except (AttributeError, OSError):
            cores = list(range(os.cpu_count() or 1))
    return [PerCoreActor(c, handler, pin) for c in cores]


# ----------------------------------------------------------------------------- connection pool

class ConnectionPool:
    """Bounded pool of reusable connections made by ``factory()``. ``acquire`` reuses an
    idle connection that passes ``check`` (and is younger than ``max_idle_s``), makes a
    new one while under ``max_size``, else waits up to ``timeout``. Use as
    ``with pool.connection() as c: ...``."""

    def __init__(self, factory: Callable[[], Any], max_size: int = 16, max_idle_s: float = 300.0,
                 check: Callable[[Any], bool] | None = None, close: Callable[[Any], None] | None = None):
        self.factory, self.max_size, self.max_idle_s = factory, max_size, max_idle_s
        self.check = check or (lambda c: True)
        self.close_fn = close or (lambda c: getattr(c, "close", lambda: None)())
        self._idle: list[tuple[float, Any]] = []
        self._out = 0
        self._cv = threading.Condition()
        self.created = self.reused = self.discarded = 0

    def acquire(self, timeout: float | None = 10.0):
        end = None if timeout is None else time.monotonic() + timeout
        with self._cv:
            while True:
                while self._idle:
                    t, c = self._idle.pop()
                    if time.monotonic() - t <= self.max_idle_s and self.check(c):
                        self._out += 1
                        self.reused += 1
                        return c
                    self.discarded += 1
                    self.close_fn(c)
                if self._out < self.max_size:
                    self._out += 1
                    break
                left = None if end is None else end - time.monotonic()
                if left is not None and left <= 0:
                    raise TimeoutError("connection pool exhausted")
                self._cv.wait(left)
        try:
            c = self.factory()
        except BaseException:
            with self._cv:
                self._out -= 1
                self._cv.notify()
            raise
        self.created += 1
        return c

    def release(self, c, broken: bool = False):
        with self._cv:
            self._out -= 1
            if broken:
                self.discarded += 1
                self.close_fn(c)
            else:
                self._idle.append((time.monotonic(), c))
            self._cv.notify()

    class _Lease:
        def __init__(self, pool):
            self.pool, self.c = pool, None

        def __enter__(self):
            self.c = self.pool.acquire()
            return self.c

        def __exit__(self, et, ev, tb):
            self.pool.release(self.c, broken=et is not None)
            return False

    def connection(self):
        return ConnectionPool._Lease(self)

    def stats(self) -> dict:
        with self._cv:
            return {"idle": len(self._idle), "in_use": self._out, "created": self.created,
                    "reused": self.reused, "discarded": self.discarded, "max_size": self.max_size}

    def close(self):
        with self._cv:
            for _, c in self._idle:
                self.close_fn(c)
            self._idle.clear()
