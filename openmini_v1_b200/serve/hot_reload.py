"""Hot model reload with two model slots (active / standby).

Reference behaviour (openmini-server/src/service/hot_reload.rs:86-224): a
double buffer of model slots; ``preload_standby`` loads a new model into the
idle slot while the active one keeps serving, ``switch_to_standby`` swaps them
atomically and notifies waiters, ``rollback`` swaps back.

Here a slot holds an ``LLMEngine``. Loading runs on a background thread (the
loader is any callable returning an engine, e.g. a GGUF load onto the GPU).
The switch waits until the active engine has no request in flight, or moves
its unfinished requests to the new engine when ``migrate=True`` (their token
ids are re-prefilled there), so no request is lost. ``engine()`` always returns
the current active engine; callers hold no reference across steps.
"""
from __future__ import annotations

import threading
import time
from dataclasses import dataclass


@dataclass
class SlotInfo:
    name: str = ""
    version: int = 0
    loaded_at: float = 0.0


class HotReloader:
    def __init__(self, engine, name: str = "initial"):
        self._slots = [engine, None]
        self._info = [SlotInfo(name, 1, time.time()), SlotInfo()]
        self._active = 0
        self._lock = threading.Lock()
        self._switched = threading.Condition(self._lock)
        self._loading: threading.Thread | None = None
        self.load_error: BaseException | None = None
        self.version = 1

    # ------------------------------------------------------------------ state
    def engine(self):
        with self._lock:
            return self._slots[self._active]

    def status(self) -> dict:
        with self._lock:
            a, s = self._active, 1 - self._active
            return {"active": vars(self._info[a]).copy(), "standby": vars(self._info[s]).copy(),
                    "standby_ready": self._slots[s] is not None,
                    "loading": self._loading is not None and self._loading.is_alive(),
                    "error": repr(self.load_error) if self.load_error else None}

    # ------------------------------------------------------------------ load
    def preload_standby(self, loader, name: str, block: bool = False):
        """Build the standby engine with ``loader()`` on a background thread."""
        if self._loading is not None and self._loading.is_alive():
            raise RuntimeError("a standby load is already running")
        self.load_error = None

        def run():
            try:
                eng = loader()
            except BaseException as e:  # reported through status()
                self.load_error = e
                return
            with self._lock:
                s = 1 - self._active
                self._slots[s] = eng
                self._info[s] = SlotInfo(name, self.version + 1, time.time())

        self._loading = threading.Thread(target=run, daemon=True, name="openmini-hot-reload")
        self._loading.start()
        if block:
            self._loading.join()
            if self.load_error:
                raise self.load_error

    def wait_standby(self, timeout: float | None = None) -> bool:
        if self._loading is not None:
            self._loading.join(timeout)
        with self._lock:
            return self._slots[1 - self._active] is not None

    # ------------------------------------------------------------------ switch
    def switch_to_standby(self, migrate: bool = True, drain_timeout: float = 30.0) -> int:
        """Make the standby engine active. Unfinished requests move to it (``migrate``)
        or the switch waits for them to drain. Returns the new version."""
        with self._lock:
            s = 1 - self._active
            new = self._slots[s]
            if new is None:
                raise RuntimeError("no standby model loaded")
            old = self._slots[self._active]
        if migrate:
            for r in old.take_unfinished():
                new.adopt(r)
        else:
            t0 = time.monotonic()
            while old.has_unfinished() and time.monotonic() - t0 < drain_timeout:
                old.step()
        with self._lock:
            self._active = s
            self.version = self._info[s].version
            self._switched.notify_all()
            return self.version

    def rollback(self) -> int:
        """Swap back to the previous engine (if it is still held)."""
        with self._lock:
            if self._slots[1 - self._active] is None:
                raise RuntimeError("nothing to roll back to")
            self._active = 1 - self._active
            self.version = self._info[self._active].version
            self._switched.notify_all()
            return self.version

    def release_standby(self):
        with self._lock:
            self._slots[1 - self._active] = None
            self._info[1 - self._active] = SlotInfo()

    def wait_switch(self, version: int, timeout: float | None = None) -> bool:
        with self._lock:
            return self._switched.wait_for(lambda: self.version >= version, timeout)
