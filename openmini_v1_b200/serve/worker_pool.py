"""Multi-process worker pool with the reference's pipe protocol
(openmini-server/src/service/worker/pool.rs:82-560, worker.rs:36-283):
workers are child processes talking over stdin/stdout with command bytes
{1 TASK, 2 SHUTDOWN, 3 HEARTBEAT, 4 LOAD_MODEL} and little-endian
length-prefixed Task / TaskResult frames (encoded by the C++ runtime).

Dispatch is round-robin over idle workers; a heartbeat thread pings every
worker, marks it dead when it misses the deadline or its process exits, and
restarts it when ``restart_on_failure`` is set. Tasks in flight on a dead
worker fail with an error result (no silent loss).

A worker runs ``python -m openmini_v1_b200.serve.worker_main <handler>``
where ``<handler>`` is "module:function" mapping task bytes -> result bytes.
"""
from __future__ import annotations

import os
import struct
import subprocess
import sys
import threading
import time

from .. import _native

IDLE, BUSY, DEAD = 0, 1, 2


def _read_exact(f, n):
    buf = b""
    while len(buf) < n:
        chunk = f.read(n - len(buf))
        if not chunk:
            raise EOFError("worker pipe closed")
        buf += chunk
    return buf


class WorkerHandle:
    def __init__(self, wid: int, handler: str, env=None):
        self.id = wid
        self.handler = handler
        e = dict(os.environ)
        e.update(env or {})
        e["MINICPM_WORKER_ID"] = str(wid)
        e["OPENMINI_WORKER_ID"] = str(wid)
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        e["PYTHONPATH"] = root + os.pathsep + e.get("PYTHONPATH", "")
        self.proc = subprocess.Popen([sys.executable, "-m", "openmini_v1_b200.serve.worker_main", handler],
                                     stdin=subprocess.PIPE, stdout=subprocess.PIPE, env=e)
        self.state = IDLE
        self.last_heartbeat = time.time()
        self.lock = threading.Lock()
        self.tasks_done = 0

    @property
    def pid(self):
        return self.proc.pid

    def alive(self) -> bool:
        return self.proc.poll() is None and self.state != DEAD

    def _send(self, b: bytes):
        self.proc.stdin.write(b)
        self.proc.stdin.flush()

    def run_task(self, task_id: int, data: bytes, timeout: float):
        rt = _native.rt()
        with self.lock:
            self.state = BUSY
            try:
                self._send(rt.encode_command(rt.WORKER_CMD_TASK, rt.encode_task(task_id, data)))
                n = struct.unpack("<I", _read_exact(self.proc.stdout, 4))[0]
                tid, ok, payload = rt.decode_result(_read_exact(self.proc.stdout, n))
                self.tasks_done += 1
                self.state = IDLE
                return tid, ok, payload
            except (EOFError, BrokenPipeError, OSError) as e:
                self.state = DEAD
                return task_id, False, f"worker {self.id} failed: {e}".encode()

    def heartbeat(self, timeout: float) -> bool:
        if self.state == BUSY:  # busy workers prove liveness by finishing tasks; check the process only
            return self.proc.poll() is None
        if not self.lock.acquire(timeout=timeout):
            return self.proc.poll() is None
        try:
            rt = _native.rt()
            self._send(rt.encode_command(rt.WORKER_CMD_HEARTBEAT))
            ok = _read_exact(self.proc.stdout, 1) == b"\x03"
            if ok:
                self.last_heartbeat = time.time()
            return ok
        except (EOFError, BrokenPipeError, OSError):
            return False
        finally:
            self.lock.release()

    def shutdown(self, timeout: float = 5.0):
        try:
            self._send(_native.rt().encode_command(_native.rt().WORKER_CMD_SHUTDOWN))
        except (BrokenPipeError, OSError):
            pass
        try:
            self.proc.wait(timeout)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()

    def kill(self):
        self.proc.kill()
        self.proc.wait()


class WorkerPool:
    def __init__(self, count: int, handler: str, restart_on_failure: bool = True,
                 health_check_interval_ms: int = 5000, task_timeout_s: float = 300.0):
        self.handler = handler
        self.restart = restart_on_failure
        self.timeout = task_timeout_s
        self.interval = health_check_interval_ms / 1000.0
        self.workers = [WorkerHandle(i, handler) for i in range(count)]
        self.rr = 0
        self.lock = threading.Lock()
        self.next_task = 1
        self.restarts = 0
        self._stop = threading.Event()
        self._hb = threading.Thread(target=self._health_loop, daemon=True)
        self._hb.start()

    def _pick(self):
        with self.lock:
            n = len(self.workers)
            for k in range(n):
                w = self.workers[(self.rr + k) % n]
                if w.alive() and w.state == IDLE:
                    self.rr = (self.rr + k + 1) % n
                    return w
            live = [w for w in self.workers if w.alive()]
            if not live:
                return None
            w = live[self.rr % len(live)]
            self.rr += 1
            return w

    def dispatch(self, data: bytes):
        """Run one task; returns (ok, payload)."""
        w = self._pick()
        if w is None:
            return False, b"no live workers"
        with self.lock:
            tid = self.next_task
            self.next_task += 1
        _, ok, payload = w.run_task(tid, data, self.timeout)
        if w.state == DEAD:
            self._replace(w)
        return ok, payload

    def _replace(self, w):
        if not self.restart:
            return
        with self.lock:
            if w in self.workers and w.state == DEAD or (w in self.workers and w.proc.poll() is not None):
                i = self.workers.index(w)
                try:
                    w.kill()
                except Exception:
                    pass
                self.workers[i] = WorkerHandle(w.id, self.handler)
                self.restarts += 1

    def health_check(self) -> dict:
        status = {}
        for w in list(self.workers):
            ok = w.alive() and w.heartbeat(timeout=self.interval)
            if not ok:
                w.state = DEAD
                self._replace(w)
            status[w.id] = ok
        return status

    def _health_loop(self):
        while not self._stop.wait(self.interval):
            self.health_check()

    def stats(self) -> dict:
        return {"workers": len(self.workers), "alive": sum(w.alive() for w in self.workers),
                "restarts": self.restarts, "tasks_done": sum(w.tasks_done for w in self.workers)}

    def shutdown(self):
        self._stop.set()
        for w in self.workers:
            w.shutdown()
