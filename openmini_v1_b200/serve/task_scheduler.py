"""Task scheduling front-ends of the reference's service layer.

``TaskScheduler`` (openmini-server/src/service/scheduler/mod.rs:228-630): a
bounded queue drained by ``max_concurrent`` workers, with submit / status /
shutdown and per-task timeouts. ``AsyncInferencePool``
(openmini-server/src/service/worker/async_pool.rs:13-181): collects up to
``batch_size`` tasks or waits ``batch_timeout`` and hands the batch to one
``engine_fn(list) -> list`` call, replying to each submitter. In this
framework both wrap real work (engine requests, worker-pool dispatch); the
reference's task bodies were placeholders.
"""
from __future__ import annotations

import asyncio
import enum
import itertools
import time


class TaskStatus(enum.Enum):
    QUEUED = "queued"
    RUNNING = "running"
    DONE = "done"
    FAILED = "failed"
    TIMEOUT = "timeout"


class QueueFull(Exception):
    pass


class TaskScheduler:
    def __init__(self, max_concurrent: int = 4, queue_capacity: int = 1000, task_timeout_s: float = 300.0):
        self.max_concurrent = max_concurrent
        self.queue: asyncio.Queue | None = None
        self.capacity = queue_capacity
        self.timeout = task_timeout_s
        self.status: dict = {}
        self.results: dict = {}
        self._ids = itertools.count(1)
        self._workers = []
        self._running = False
        self.completed = 0
        self.failed = 0

    async def start(self):
        self.queue = asyncio.Queue(self.capacity)
        self._running = True
        self._workers = [asyncio.create_task(self._worker()) for _ in range(self.max_concurrent)]

    async def _worker(self):
        while self._running:
            tid, fn, fut = await self.queue.get()
            self.status[tid] = TaskStatus.RUNNING
            try:
                res = await asyncio.wait_for(fn(), self.timeout)
                self.status[tid] = TaskStatus.DONE
                self.completed += 1
                if not fut.done():
                    fut.set_result(res)
            except asyncio.TimeoutError:
                self.status[tid] = TaskStatus.TIMEOUT
                self.failed += 1
                if not fut.done():
                    fut.set_exception(TimeoutError(f"task {tid} timed out"))
            except Exception as e:
                self.status[tid] = TaskStatus.FAILED
                self.failed += 1
                if not fut.done():
                    fut.set_exception(e)
            finally:
                self.queue.task_done()

    def submit(self, fn) -> tuple:
        """Queue ``fn`` (an async callable); returns (task id, future). Raises QueueFull."""
        if not self._running:
            raise RuntimeError("scheduler not started")
        tid = next(self._ids)
        fut = asyncio.get_running_loop().create_future()
        try:
            self.queue.put_nowait((tid, fn, fut))
        except asyncio.QueueFull:
            raise QueueFull(f"queue capacity {self.capacity} reached")
        self.status[tid] = TaskStatus.QUEUED
        return tid, fut

    def get_status(self, tid) -> TaskStatus | None:
        return self.status.get(tid)

    def stats(self) -> dict:
        return {"queued": self.queue.qsize() if self.queue else 0, "completed": self.completed,
                "failed": self.failed, "max_concurrent": self.max_concurrent}

    async def shutdown(self, drain: bool = True):
        if drain and self.queue is not None:
            await self.queue.join()
        self._running = False
        for w in self._workers:
            w.cancel()
        await asyncio.gather(*self._workers, return_exceptions=True)


class AsyncInferencePool:
    def __init__(self, engine_fn, batch_size: int = 8, batch_timeout_ms: int = 5, request_timeout_s: float = 300.0):
        self.engine_fn = engine_fn
        self.batch_size = batch_size
        self.batch_timeout = batch_timeout_ms / 1000.0
        self.request_timeout = request_timeout_s
        self.queue: asyncio.Queue | None = None
        self._task = None
        self.batches = 0

    async def start(self):
        self.queue = asyncio.Queue()
        self._task = asyncio.create_task(self._batch_loop())

    async def _batch_loop(self):
        while True:
            first = await self.queue.get()
            batch = [first]
            deadline = time.monotonic() + self.batch_timeout
            while len(batch) < self.batch_size:
                left = deadline - time.monotonic()
                if left <= 0:
                    break
                try:
                    batch.append(await asyncio.wait_for(self.queue.get(), left))
                except asyncio.TimeoutError:
                    break
            self.batches += 1
            tasks = [t for t, _ in batch]
            try:
                res = self.engine_fn(tasks)
                if asyncio.iscoroutine(res):
                    res = await res
                for (_, fut), r in zip(batch, res):
                    if not fut.done():
                        fut.set_result(r)
            except Exception as e:
                for _, fut in batch:
                    if not fut.done():
                        fut.set_exception(e)

    async def submit(self, task):
        fut = asyncio.get_running_loop().create_future()
        await self.queue.put((task, fut))
        return await asyncio.wait_for(fut, self.request_timeout)

    async def shutdown(self):
        if self._task:
            self._task.cancel()
            await asyncio.gather(self._task, return_exceptions=True)
