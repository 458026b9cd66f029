"""Dynamic parallel-strategy adjustment and device discovery for multi-node serving.

``DynamicAdjuster`` watches serving metrics and re-plans the (tp, pp, dp) layout:
  * bottleneck detection: memory (KV or weights near the budget), communication
    (collective time share above a bound), compute / bandwidth (a step far above the
    bandwidth model), latency (SLA misses), errors;
  * candidates: every feasible (tp, pp) of the GPU count, scored with the decode
    bandwidth model (``cluster.estimate_decode_tok_s``) and a penalty for the
    communication the bottleneck reports;
  * guarded switching: a minimum number of samples, a cooldown after each change,
    a minimum predicted gain, and a rollback when the observed score after a switch
    falls below the score before it.
``Discovery`` announces this node over UDP (broadcast or a static peer list) and keeps
a registry of peers with their resources, marking them lost after ``timeout_s``
without an announcement; callers get join / leave / update events.

Reference counterparts: openmini-server/src/distributed/exo_dynamic_adjuster.rs
(PerformanceMetrics, BottleneckType, AdjustmentDecision, rollback) and
distributed/discovery.rs (ExoDeviceDiscovery, PeerRegistry, DiscoveryEvent).
"""
from __future__ import annotations

import json
import socket
import statistics
import threading
import time
from dataclasses import asdict, dataclass, field

from .cluster import ModelSpec, Plan, estimate_decode_tok_s, make_plan, plan_parallelism


@dataclass
class PerformanceMetrics:
    p50_ms: float
    p99_ms: float
    throughput_tps: float
    gpu_util: float = 0.0          # 0..1
    mem_util: float = 0.0          # 0..1 of the device
    comm_frac: float = 0.0         # share of the step in collectives
    error_rate: float = 0.0
    t: float = field(default_factory=time.time)

    def score(self) -> float:
        """Higher is better: throughput, discounted by tail latency and errors."""
        return self.throughput_tps / (1.0 + self.p99_ms / 1000.0) * (1.0 - min(self.error_rate, 1.0))

    def meets_sla(self, p99_ms: float, min_tps: float) -> bool:
        return self.p99_ms <= p99_ms and self.throughput_tps >= min_tps


BOTTLENECKS = ("none", "memory", "communication", "compute", "latency", "errors")


@dataclass
class Decision:
    action: str                 # keep | switch | rollback
    plan: Plan | None
    bottleneck: str
    predicted_gain: float = 0.0
    reason: str = ""
    t: float = field(default_factory=time.time)


@dataclass
class AdjusterConfig:
    sla_p99_ms: float = 2000.0
    min_tps: float = 0.0
    mem_high: float = 0.92
    comm_high: float = 0.25
    min_samples: int = 5
    cooldown_s: float = 60.0
    min_gain: float = 0.10
    rollback_margin: float = 0.05


class DynamicAdjuster:
    def __init__(self, spec: ModelSpec, gpus: int, batch: int, cfg: AdjusterConfig | None = None,
                 gpu_mem_gb: float = 180.0, clock=time.time):
        self.spec, self.gpus, self.batch = spec, gpus, batch
        self.cfg = cfg or AdjusterConfig()
        self.mem = gpu_mem_gb
        self.clock = clock
        self.current = plan_parallelism(spec, gpus, gpu_mem_gb)
        self.history: list[PerformanceMetrics] = []
        self.decisions: list[Decision] = []
        self._last_switch = -1e18
        self._before: tuple | None = None   # (plan, score) before the last switch

    def record(self, m: PerformanceMetrics):
        self.history = (self.history + [m])[-256:]

    def _recent(self):
        return self.history[-self.cfg.min_samples:]

    def bottleneck(self) -> str:
        r = self._recent()
        if not r:
            return "none"
        med = lambda f: statistics.median(f(x) for x in r)  # noqa: E731
        if med(lambda x: x.error_rate) > 0.05:
            return "errors"
        if med(lambda x: x.mem_util) >= self.cfg.mem_high:
            return "memory"
        if med(lambda x: x.comm_frac) >= self.cfg.comm_high:
            return "communication"
        if med(lambda x: x.p99_ms) > self.cfg.sla_p99_ms:
            return "latency"
        if med(lambda x: x.gpu_util) >= 0.9:
            return "compute"
        return "none"

    def candidates(self) -> list[Plan]:
        """Every (tp <= 8, pp) layout that divides the GPUs and fits in memory."""
        out = []
        tp = 1
        while tp <= min(8, self.gpus):
            for pp in range(1, self.gpus // tp + 1):
                if self.gpus % (tp * pp) == 0:
                    p = make_plan(self.spec, tp, pp, self.gpus, self.mem)
                    if p.fits:
                        out.append(p)
            tp *= 2
        return out or [self.current]

    def _predict(self, plan: Plan, bottleneck: str) -> float:
        tps = estimate_decode_tok_s(self.spec, plan, self.batch)
        if bottleneck == "communication":  # collectives scale with the TP degree (and PP hops)
            tps /= 1.0 + 0.1 * (plan.tp - 1) + 0.05 * (plan.pp - 1)
        if bottleneck == "memory":         # headroom matters more than raw speed
            tps *= 1.0 if plan.weight_gb_per_gpu + plan.kv_gb_per_gpu < self.mem * self.cfg.mem_high else 0.5
        return tps

    def evaluate(self) -> Decision:
        now = self.clock()
        r = self._recent()
        if len(r) < self.cfg.min_samples:
            return self._log(Decision("keep", self.current, "none", reason="not enough samples"))
        score = statistics.median(x.score() for x in r)
        if self._before is not None:  # judge the last switch
            prev_plan, prev_score = self._before
            self._before = None
            if score < prev_score * (1 - self.cfg.rollback_margin):
                self.current = prev_plan
                self._last_switch = now
                self.history.clear()
                return self._log(Decision("rollback", prev_plan, "none",
                                          reason=f"score {score:.1f} < {prev_score:.1f} before the switch"))
        b = self.bottleneck()
        if b == "none" or now - self._last_switch < self.cfg.cooldown_s:
            return self._log(Decision("keep", self.current, b, reason="no bottleneck" if b == "none" else "cooldown"))
        base = self._predict(self.current, b)
        best, gain = self.current, 0.0
        for p in self.candidates():
            g = self._predict(p, b) / base - 1.0 if base > 0 else 0.0
            if (p.tp, p.pp) != (self.current.tp, self.current.pp) and g > gain:
                best, gain = p, g
        if gain < self.cfg.min_gain:
            return self._log(Decision("keep", self.current, b, gain, "no candidate clears the minimum gain"))
        self._before = (self.current, score)
        self.current = best
        self._last_switch = now
        self.history.clear()
        return self._log(Decision("switch", best, b, gain, best.reason))

    def _log(self, d: Decision) -> Decision:
        self.decisions.append(d)
        return d


# ----------------------------------------------------------------------------- discovery

@dataclass
class PeerInfo:
    node_id: str
    address: str
    gpus: int
    gpu_mem_gb: float
    load: float = 0.0
    last_seen: float = 0.0
    alive: bool = True


class Discovery:
    """Announces ``info`` every ``interval_s`` to ``peers`` (list of (host, port)) or to the
    UDP broadcast address, and listens on ``port`` for the announcements of others."""

    def __init__(self, info: PeerInfo, port: int, peers: list | None = None, interval_s: float = 0.2,
                 timeout_s: float = 1.0, on_event=None):
        self.info, self.port, self.peers = info, port, peers
        self.interval, self.timeout = interval_s, timeout_s
        self.on_event = on_event or (lambda kind, peer: None)
        self.registry: dict[str, PeerInfo] = {}
        self.events: list[tuple] = []
        self._stop = threading.Event()
        self._rx = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
        self._rx.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self._rx.bind(("0.0.0.0" if peers is None else "127.0.0.1", port))
        self._rx.settimeout(0.05)
        self._tx = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
        if peers is None:
            self._tx.setsockopt(socket.SOL_SOCKET, socket.SO_BROADCAST, 1)
        self._threads = [threading.Thread(target=f, daemon=True) for f in (self._announce, self._listen)]

    def start(self):
        for t in self._threads:
            t.start()
        return self

    def stop(self):
        self._stop.set()
        for t in self._threads:
            t.join(2)
        self._rx.close()
        self._tx.close()

    def _emit(self, kind, peer):
        self.events.append((kind, peer.node_id))
        self.on_event(kind, peer)

    def _announce(self):
        while not self._stop.is_set():
            msg = json.dumps({"om": 1, **asdict(self.info)}).encode()
            for dst in (self.peers if self.peers is not None else [("255.255.255.255", self.port)]):
                try:
                    self._tx.sendto(msg, dst)
                except OSError:
                    pass
            self._expire()
            self._stop.wait(self.interval)

    def _listen(self):
        while not self._stop.is_set():
            try:
                data, _ = self._rx.recvfrom(65536)
            except (socket.timeout, OSError):
                continue
            try:
                d = json.loads(data)
            except ValueError:
                continue
            if d.pop("om", None) != 1 or d.get("node_id") == self.info.node_id:
                continue
            d["last_seen"], d["alive"] = time.monotonic(), True
            peer = PeerInfo(**d)
            old = self.registry.get(peer.node_id)
            self.registry[peer.node_id] = peer
            if old is None or not old.alive:
                self._emit("joined", peer)
            elif (old.gpus, old.gpu_mem_gb, old.address) != (peer.gpus, peer.gpu_mem_gb, peer.address):
                self._emit("updated", peer)

    def _expire(self):
        now = time.monotonic()
        for p in list(self.registry.values()):
            if p.alive and now - p.last_seen > self.timeout:
                p.alive = False
                self._emit("left", p)

    def alive(self) -> list[PeerInfo]:
        return [p for p in self.registry.values() if p.alive]

    def total_gpus(self) -> int:
        return self.info.gpus + sum(p.gpus for p in self.alive())
