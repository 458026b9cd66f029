"""Component health, readiness and liveness.

Components: gpu (device memory use, kernel status word, NVML temperature when
available), memory (host), cpu (load average), scheduler (queue length) and
model (weights loaded). Each is healthy / degraded / unhealthy against the
reference's default thresholds (HealthCheckerConfig: GPU 80/95 %, memory
80/90 %, CPU 85 %, queue 50; openmini-server/src/monitoring/
health_check.rs:125-363). Routes: /health/ready, /health/live, /health/model,
/health/components.
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field


@dataclass
class HealthConfig:
    gpu_warning: float = 80.0
    gpu_error: float = 95.0
    memory_warning: float = 80.0
    memory_error: float = 90.0
    cpu_warning: float = 85.0
    queue_warning: int = 50


@dataclass
class Component:
    name: str
    status: str = "healthy"    # healthy | degraded | unhealthy
    message: str = ""
    details: dict = field(default_factory=dict)


def _host_mem_pct() -> float:
    tot = avail = 0
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemTotal:"):
                    tot = int(line.split()[1])
                elif line.startswith("MemAvailable:"):
                    avail = int(line.split()[1])
    except OSError:
        return 0.0
    return 100.0 * (tot - avail) / tot if tot else 0.0


class HealthChecker:
    def __init__(self, engine=None, cfg: HealthConfig | None = None, model_loaded=lambda: True):
        self.engine = engine
        self.cfg = cfg or HealthConfig()
        self.model_loaded = model_loaded
        self.started = time.time()

    def _grade(self, c: Component, v: float, warn: float, err: float | None = None):
        if err is not None and v >= err:
            c.status = "unhealthy"
        elif v >= warn:
            c.status = "degraded"

    def check_gpu(self) -> Component:
        c = Component("gpu")
        try:
            import torch
            if not torch.cuda.is_available():
                c.details["available"] = False
                return c
            free, total = torch.cuda.mem_get_info()
            pct = 100.0 * (total - free) / total
            c.details.update(used_pct=round(pct, 1), total_bytes=total)
            self._grade(c, pct, self.cfg.gpu_warning, self.cfg.gpu_error)
            from .. import ops
            st = int(ops.ctx(torch.device("cuda", torch.cuda.current_device())).status.item())
            c.details["kernel_status"] = st
            if st != 0:
                c.status, c.message = "unhealthy", f"a device wait gave up (status {st})"
        except Exception as e:  # health must answer even when the device does not
            c.status, c.message = "unhealthy", repr(e)
        return c

    def check_memory(self) -> Component:
        c = Component("memory")
        pct = _host_mem_pct()
        c.details["used_pct"] = round(pct, 1)
        self._grade(c, pct, self.cfg.memory_warning, self.cfg.memory_error)
        return c

    def check_cpu(self) -> Component:
        c = Component("cpu")
        try:
            load = os.getloadavg()[0] / max(os.cpu_count() or 1, 1) * 100.0
        except OSError:
            load = 0.0
        c.details["load_pct"] = round(load, 1)
        self._grade(c, load, self.cfg.cpu_warning)
        return c

    def check_scheduler(self) -> Component:
        c = Component("scheduler")
        if self.engine is not None:
            e = getattr(self.engine, "engine", self.engine)
            q = len(getattr(e.sched, "waiting", []))
            c.details.update(waiting=q, running=len(getattr(e.sched, "running", [])))
            self._grade(c, q, self.cfg.queue_warning)
        return c

    def check_model(self) -> Component:
        c = Component("model")
        if not self.model_loaded():
            c.status, c.message = "unhealthy", "model not loaded"
        return c

    def check(self) -> dict:
        comps = [self.check_gpu(), self.check_memory(), self.check_cpu(), self.check_scheduler(), self.check_model()]
        worst = "healthy"
        for c in comps:
            if c.status == "unhealthy":
                worst = "unhealthy"
            elif c.status == "degraded" and worst == "healthy":
                worst = "degraded"
        return {"status": worst, "uptime_s": round(time.time() - self.started, 1),
                "components": [c.__dict__ for c in comps]}


def mount_health(app, checker: HealthChecker):
    from starlette.responses import JSONResponse

    @app.get("/health/live")
    async def live():
        return {"status": "alive"}

    @app.get("/health/ready")
    async def ready():
        r = checker.check()
        ok = r["status"] != "unhealthy"
        return JSONResponse({"ready": ok, **r}, status_code=200 if ok else 503)

    @app.get("/health/model")
    async def model():
        c = checker.check_model()
        return JSONResponse(c.__dict__, status_code=200 if c.status == "healthy" else 503)

    @app.get("/health/components")
    async def components():
        return checker.check()
