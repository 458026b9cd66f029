"""Memory management and load monitoring.

* :class:`MemoryMonitor` samples host RAM (``/proc/meminfo`` or psutil) and device
  HBM (``torch.cuda.mem_get_info`` plus the caching allocator's counters), classifies
  the pressure (normal / warning / critical) and calls registered callbacks when the
  level changes. The engine uses the KV budget helper to size its paged cache.
* :class:`DeviceArena` is a bump allocator over one device buffer: scratch tensors
  for a step are carved out of it with 256-byte alignment and released all at once
  with :meth:`DeviceArena.reset`, so the hot path makes no allocator calls.
* :class:`LoadMonitor` reads CPU load (``/proc/loadavg``) and, through NVML (read
  only; nothing is ever set), GPU utilisation, temperature, power and the active
  clock-event reasons.

Reference counterparts: openmini-server/src/hardware/memory/monitor.rs (pressure
levels and callbacks), hardware/memory/arena.rs and pool.rs (arena / pool
allocators), hardware/load_monitor.rs (CPU load and thermal state).
"""
from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass, field
from typing import Callable

NORMAL, WARNING, CRITICAL = "normal", "warning", "critical"


@dataclass
class MemorySnapshot:
    host_total: int
    host_available: int
    dev_total: int = 0
    dev_free: int = 0
    dev_allocated: int = 0      # bytes in live tensors (caching allocator)
    dev_reserved: int = 0       # bytes held by the caching allocator
    t: float = field(default_factory=time.monotonic)

    @property
    def host_used_frac(self) -> float:
        return 1.0 - self.host_available / self.host_total if self.host_total else 0.0

    @property
    def dev_used_frac(self) -> float:
        return 1.0 - self.dev_free / self.dev_total if self.dev_total else 0.0


def _host_mem() -> tuple[int, int]:
    try:
        info = {}
        with open("/proc/meminfo") as f:
            for line in f:
                k, v = line.split(":", 1)
                info[k] = int(v.split()[0]) * 1024
        return info["MemTotal"], info.get("MemAvailable", info.get("MemFree", 0))
    except (OSError, KeyError, ValueError):
        try:
            import psutil
            vm = psutil.virtual_memory()
            return vm.total, vm.available
        except Exception:
            return 0, 0


class MemoryMonitor:
    """Pressure thresholds are fractions of used memory (the worse of host and device)."""

    def __init__(self, device=None, warning: float = 0.85, critical: float = 0.95,
                 sampler: Callable[[], MemorySnapshot] | None = None):
        self.device = device
        self.warning, self.critical = warning, critical
        self._sampler = sampler or self._sample
        self._callbacks: list[Callable[[str, MemorySnapshot], None]] = []
        self.level = NORMAL
        self.history: list[MemorySnapshot] = []
        self._stop = threading.Event()
        self._thread = None

    def _sample(self) -> MemorySnapshot:
        tot, avail = _host_mem()
        snap = MemorySnapshot(tot, avail)
        if self.device is not None:
            import torch
            dev = torch.device(self.device)
            if dev.type == "cuda" and torch.cuda.is_available():
                free, total = torch.cuda.mem_get_info(dev)
                snap.dev_total, snap.dev_free = total, free
                snap.dev_allocated = torch.cuda.memory_allocated(dev)
                snap.dev_reserved = torch.cuda.memory_reserved(dev)
        return snap

    def on_change(self, cb: Callable[[str, MemorySnapshot], None]):
        self._callbacks.append(cb)

    def classify(self, snap: MemorySnapshot) -> str:
        used = max(snap.host_used_frac, snap.dev_used_frac)
        return CRITICAL if used >= self.critical else WARNING if used >= self.warning else NORMAL

    def poll(self) -> MemorySnapshot:
        snap = self._sampler()
        self.history = (self.history + [snap])[-256:]
        lvl = self.classify(snap)
        if lvl != self.level:
            self.level = lvl
            for cb in self._callbacks:
                cb(lvl, snap)
        return snap

    def start(self, interval_s: float = 1.0):
        def run():
            while not self._stop.wait(interval_s):
                self.poll()
        self._thread = threading.Thread(target=run, name="mem-monitor", daemon=True)
        self._thread.start()

    def stop(self):
        self._stop.set()
        if self._thread:
            self._thread.join(5)


def kv_block_budget(free_bytes: int, total_bytes: int, per_block_bytes: int, utilization: float = 0.9,
                    reserve_bytes: int = 4 << 30) -> int:
    """Paged-KV blocks that fit in ``utilization`` of the device minus a reserve for
    activations and workspaces (180 GB B200: about 140 GB of KV at 0.9 with 4 GB held back)."""
    budget = free_bytes - (1.0 - utilization) * total_bytes - reserve_bytes
    return max(0, int(budget // max(per_block_bytes, 1)))


class DeviceArena:
    """Bump allocator over one contiguous buffer (device or host). ``alloc`` returns a
    view; ``mark``/``release_to`` give nested scopes; ``reset`` frees everything. Views
    stay valid until the arena is reset past them: the caller owns that discipline."""

    ALIGN = 256

    def __init__(self, nbytes: int, device="cpu"):
        import torch
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.capacity = nbytes
        self.offset = 0
        self.peak = 0

    def alloc(self, shape, dtype):
        import torch
        n = 1
        for s in (shape if isinstance(shape, (tuple, list)) else (shape,)):
            n *= int(s)
        el = torch.empty((), dtype=dtype).element_size()
        start = -(-self.offset // self.ALIGN) * self.ALIGN
        end = start + n * el
        if end > self.capacity:
            raise MemoryError(f"arena exhausted: need {end} of {self.capacity} bytes")
        self.offset = end
        self.peak = max(self.peak, end)
        return self.buf[start:end].view(dtype).view(*(shape if isinstance(shape, (tuple, list)) else (shape,)))

    def mark(self) -> int:
        return self.offset

    def release_to(self, mark: int):
        self.offset = mark

    def reset(self):
        self.offset = 0

    @property
    def used(self) -> int:
        return self.offset


@dataclass
class LoadSnapshot:
    load1: float
    cpus: int
    gpu_util: list = field(default_factory=list)       # percent per GPU
    gpu_temp_c: list = field(default_factory=list)
    gpu_power_w: list = field(default_factory=list)
    gpu_throttle: list = field(default_factory=list)   # names of active clock-event reasons

    @property
    def cpu_load_frac(self) -> float:
        return self.load1 / max(self.cpus, 1)


# NVML clock-event reason bits (public nvml.h values)
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}


class LoadMonitor:
    """Read-only CPU / GPU load sampling. ``nvml`` may be a fake module in tests."""

    def __init__(self, nvml=None):
        self.nvml = nvml
        if self.nvml is None:
            try:
                import pynvml
                pynvml.nvmlInit()
                self.nvml = pynvml
            except Exception:
                self.nvml = None

    def sample(self) -> LoadSnapshot:
        try:
            load1 = os.getloadavg()[0]
        except OSError:
            load1 = 0.0
        snap = LoadSnapshot(load1, os.cpu_count() or 1)
        n = self.nvml
        if n is None:
            return snap
        try:
            for i in range(n.nvmlDeviceGetCount()):
                h = n.nvmlDeviceGetHandleByIndex(i)
                snap.gpu_util.append(n.nvmlDeviceGetUtilizationRates(h).gpu)
                snap.gpu_temp_c.append(n.nvmlDeviceGetTemperature(h, 0))
                snap.gpu_power_w.append(n.nvmlDeviceGetPowerUsage(h) / 1000.0)
                bits = n.nvmlDeviceGetCurrentClocksEventReasons(h) \
                    if hasattr(n, "nvmlDeviceGetCurrentClocksEventReasons") \
                    else n.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                snap.gpu_throttle.append([v for k, v in _REASONS.items() if bits & k])
        except Exception:
            pass
        return snap

    def overloaded(self, snap: LoadSnapshot, cpu_frac: float = 0.9, temp_c: float = 85.0) -> bool:
        hot = any(t >= temp_c for t in snap.gpu_temp_c)
        thermal = any(("hw_thermal_slowdown" in r or "sw_thermal_slowdown" in r) for r in snap.gpu_throttle)
        return snap.cpu_load_frac >= cpu_frac or hot or thermal
