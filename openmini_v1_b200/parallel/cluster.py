"""Multi-node serving control plane: replica routing, a coordinator / worker mesh with
heartbeat failure detection, and the parallel-strategy planner.

Reference counterparts:
  * router strategies (round robin, least loaded, weighted, latency aware) and node
    health: openmini-server/src/distributed/router.rs:48-875,
    distributed_inference_engine.rs:223-300 (select_node);
  * mesh / coordinator / worker and the message set {Heartbeat, TaskAssign,
    TaskResult, NodeRegister, Error}: openmini-server/src/service/distributed/
    {mesh.rs:23-247, coordinator.rs:25-380, worker.rs:36-380, protocol.rs:13-200};
  * topology -> TP / PP / hybrid decision with memory estimates and presets
    (7B TP2, 14B TP4, 70B TP8): distributed/exo_parallel_strategy.rs:67-1102,
    model/inference/distributed_inference_config.rs:188-228.

The reference mesh is in-process (tokio channels). Here workers are real
processes connected over TCP (``multiprocessing.connection``, authenticated),
so the heartbeat / failover path is exercised with processes that really die:
a worker that stops heartbeating for ``heartbeat_timeout_s`` is marked dead and
its in-flight tasks are re-dispatched to live workers.
"""
from __future__ import annotations

import itertools
import math
import threading
import time
from dataclasses import dataclass, field
from multiprocessing.connection import Client, Listener

# ---------------------------------------------------------------- messages
HEARTBEAT, TASK_ASSIGN, TASK_RESULT, NODE_REGISTER, ERROR, SHUTDOWN = (
    "heartbeat", "task_assign", "task_result", "node_register", "error", "shutdown")


# ---------------------------------------------------------------- routing
@dataclass
class NodeState:
    node_id: str
    weight: float = 1.0
    inflight: int = 0
    completed: int = 0
    failures: int = 0
    ewma_latency_s: float = 0.0
    last_heartbeat: float = field(default_factory=time.monotonic)
    alive: bool = True


class Router:
    """Picks a replica for each request. Strategies: ``round_robin``, ``least_loaded``,
    ``weighted`` (smooth weighted round robin) and ``latency`` (lowest EWMA latency
    x (inflight + 1))."""

    def __init__(self, strategy: str = "least_loaded", ewma: float = 0.2):
        if strategy not in ("round_robin", "least_loaded", "weighted", "latency"):
            raise ValueError(strategy)
        self.strategy = strategy
        self.ewma = ewma
        self.nodes: dict = {}
        self._rr = itertools.count()
        self._cur: dict = {}
        self._lock = threading.Lock()

    def add(self, node_id: str, weight: float = 1.0):
        with self._lock:
            self.nodes[node_id] = NodeState(node_id, weight)
            self._cur[node_id] = 0.0

    def remove(self, node_id: str):
        with self._lock:
            self.nodes.pop(node_id, None)
            self._cur.pop(node_id, None)

    def mark(self, node_id: str, alive: bool):
        with self._lock:
            if node_id in self.nodes:
                self.nodes[node_id].alive = alive

    def select(self) -> str:
        with self._lock:
            live = [n for n in self.nodes.values() if n.alive]
            if not live:
                raise RuntimeError("no live node")
            if self.strategy == "round_robin":
                n = live[next(self._rr) % len(live)]
            elif self.strategy == "least_loaded":
                n = min(live, key=lambda x: (x.inflight, x.completed))
            elif self.strategy == "weighted":
                tot = sum(x.weight for x in live)
                for x in live:
                    self._cur[x.node_id] += x.weight
                n = max(live, key=lambda x: self._cur[x.node_id])
                self._cur[n.node_id] -= tot
            else:
                n = min(live, key=lambda x: (x.ewma_latency_s or 1e-3) * (x.inflight + 1))
            n.inflight += 1
            return n.node_id

    def done(self, node_id: str, latency_s: float, ok: bool = True):
        with self._lock:
            n = self.nodes.get(node_id)
            if n is None:
                return
            n.inflight = max(0, n.inflight - 1)
            if ok:
                n.completed += 1
                n.ewma_latency_s = latency_s if n.ewma_latency_s == 0 else (
                    (1 - self.ewma) * n.ewma_latency_s + self.ewma * latency_s)
            else:
                n.failures += 1


# ---------------------------------------------------------------- coordinator / worker
class Coordinator:
    """Accepts worker registrations, dispatches tasks through the Router, collects
    results, and re-dispatches the tasks of workers that miss heartbeats."""

    def __init__(self, address=("127.0.0.1", 0), authkey: bytes = b"openmini", strategy: str = "least_loaded",
                 heartbeat_timeout_s: float = 2.0):
        self.listener = Listener(address, authkey=authkey)
        self.address = self.listener.address
        self.router = Router(strategy)
        self.timeout = heartbeat_timeout_s
        self.conns: dict = {}
        self.pending: dict = {}      # task_id -> (node_id, payload, t_sent)
        self.results: dict = {}
        self.events: list = []
        self._lock = threading.Lock()
        self._cv = threading.Condition(self._lock)
        self._stop = False
        self._ids = itertools.count()
        threading.Thread(target=self._accept, daemon=True).start()
        threading.Thread(target=self._watchdog, daemon=True).start()

    def _accept(self):
        while not self._stop:
            try:
                c = self.listener.accept()
            except OSError:
                return
            threading.Thread(target=self._serve, args=(c,), daemon=True).start()

    def _serve(self, conn):
        node = None
        try:
            while not self._stop:
                msg = conn.recv()
                kind = msg["type"]
                if kind == NODE_REGISTER:
                    node = msg["node_id"]
                    with self._lock:
                        self.conns[node] = conn
                        self.router.add(node, msg.get("weight", 1.0))
                        self.events.append(("register", node))
                        self._cv.notify_all()
                elif kind == HEARTBEAT:
                    with self._lock:
                        if node in self.router.nodes:
                            self.router.nodes[node].last_heartbeat = time.monotonic()
                elif kind in (TASK_RESULT, ERROR):
                    with self._lock:
                        tid = msg["task_id"]
                        ent = self.pending.pop(tid, None)
                        if ent is not None:
                            self.router.done(node, time.monotonic() - ent[2], ok=kind == TASK_RESULT)
                            self.results[tid] = msg
                            self._cv.notify_all()
        except (EOFError, OSError):
            pass
        if node is not None:
            self._fail(node, "connection lost")

    def _fail(self, node, why):
        with self._lock:
            if node not in self.conns:
                return
            self.conns.pop(node, None)
            self.router.mark(node, False)
            self.events.append(("dead", node, why))
            lost = [(tid, ent) for tid, ent in self.pending.items() if ent[0] == node]
        for tid, (_, payload, _) in lost:  # fail over to the live workers
            with self._lock:
                self.pending.pop(tid, None)
            self._send(tid, payload)

    def _watchdog(self):
        while not self._stop:
            time.sleep(self.timeout / 4)
            now = time.monotonic()
            with self._lock:
                stale = [n.node_id for n in self.router.nodes.values()
                         if n.alive and now - n.last_heartbeat > self.timeout]
            for n in stale:
                self._fail(n, "heartbeat timeout")

    def _send(self, tid, payload):
        while True:
            with self._lock:
                node = self.router.select()
                conn = self.conns.get(node)
                self.pending[tid] = (node, payload, time.monotonic())
            try:
                conn.send({"type": TASK_ASSIGN, "task_id": tid, "payload": payload})
                return node
            except (OSError, AttributeError):
                self._fail(node, "send failed")

    def wait_workers(self, n: int, timeout: float = 30.0) -> bool:
        with self._lock:
            return self._cv.wait_for(lambda: sum(1 for x in self.router.nodes.values() if x.alive) >= n, timeout)

    def submit(self, payload) -> int:
        tid = next(self._ids)
        self._send(tid, payload)
        return tid

    def collect(self, tids, timeout: float = 60.0) -> dict:
        with self._lock:
            ok = self._cv.wait_for(lambda: all(t in self.results for t in tids), timeout)
            if not ok:
                raise TimeoutError(f"{sum(t not in self.results for t in tids)} tasks unfinished")
            return {t: self.results[t] for t in tids}

    def shutdown(self):
        self._stop = True
        with self._lock:
            conns = list(self.conns.values())
        for c in conns:
            try:
                c.send({"type": SHUTDOWN})
            except OSError:
                pass
        self.listener.close()


def run_worker(address, node_id: str, handler, authkey: bytes = b"openmini", heartbeat_s: float = 0.25,
               weight: float = 1.0):
    """Worker loop: register, heartbeat on a thread, run ``handler(payload)`` per task."""
    conn = Client(address, authkey=authkey)
    lock = threading.Lock()
    stop = threading.Event()

    def send(m):
        with lock:
            conn.send(m)

    send({"type": NODE_REGISTER, "node_id": node_id, "weight": weight})

    def beat():
        while not stop.is_set():
            try:
                send({"type": HEARTBEAT, "node_id": node_id, "t": time.time()})
            except OSError:
                return
            stop.wait(heartbeat_s)

    threading.Thread(target=beat, daemon=True).start()
    try:
        while True:
            msg = conn.recv()
            if msg["type"] == SHUTDOWN:
                break
            if msg["type"] == TASK_ASSIGN:
                try:
                    send({"type": TASK_RESULT, "task_id": msg["task_id"], "node_id": node_id,
                          "result": handler(msg["payload"])})
                except Exception as e:  # reported, the worker stays up
                    send({"type": ERROR, "task_id": msg["task_id"], "node_id": node_id, "error": repr(e)})
    except (EOFError, OSError):
        pass
    finally:
        stop.set()
        conn.close()


# ---------------------------------------------------------------- strategy planner
@dataclass
class ModelSpec:
    params_b: float            # parameters, billions
    layers: int
    hidden: int
    kv_heads: int
    head_dim: int
    bytes_per_param: float = 2.0


@dataclass
class Plan:
    tp: int
    pp: int
    dp: int
    weight_gb_per_gpu: float
    kv_gb_per_gpu: float
    fits: bool
    reason: str


PRESETS = {  # name -> (ModelSpec, default tp, pp)
    "llama-7b": (ModelSpec(6.7, 32, 4096, 32, 128), 2, 1),
    "dsa-14b": (ModelSpec(14.8, 40, 5120, 8, 128), 4, 1),
    "llama-70b": (ModelSpec(70.6, 80, 8192, 8, 128), 8, 1),
}


def make_plan(spec: ModelSpec, tp: int, pp: int, gpus: int, gpu_mem_gb: float = 180.0,
              kv_tokens: int = 256 * 4608, mem_util: float = 0.9, kv_bytes: int = 2) -> Plan:
    """The memory footprint of one given (tp, pp) layout on ``gpus`` GPUs."""
    kv_per_token = 2 * spec.layers * spec.kv_heads * spec.head_dim * kv_bytes
    w = spec.params_b * spec.bytes_per_param / (tp * pp)
    kv = kv_tokens * kv_per_token / 1e9 / (tp * pp)
    ok = w + kv <= gpu_mem_gb * mem_util
    return Plan(tp, pp, max(1, gpus // (tp * pp)), w, kv, ok,
                f"tp{tp} pp{pp} dp{max(1, gpus // (tp * pp))}" + ("" if ok else ": does not fit"))


def plan_parallelism(spec: ModelSpec, gpus: int, gpu_mem_gb: float = 180.0, nvlink_domain: int = 8,
                     kv_tokens: int = 256 * 4608, mem_util: float = 0.9, kv_bytes: int = 2) -> Plan:
    """Smallest TP (a power of two within one NVLink domain, dividing the KV heads when
    possible) whose weights + KV fit; PP across domains when one domain is not enough;
    the remaining GPUs become data-parallel replicas."""
    kv_per_token = 2 * spec.layers * spec.kv_heads * spec.head_dim * kv_bytes
    budget = gpu_mem_gb * mem_util
    weights = spec.params_b * spec.bytes_per_param
    kv_total = kv_tokens * kv_per_token / 1e9
    max_tp = min(nvlink_domain, gpus)

    def fits(tp, pp):
        return weights / (tp * pp) + kv_total / (tp * pp) <= budget

    def plan(tp, pp, ok, why):
        return Plan(tp, pp, max(1, gpus // (tp * pp)), weights / (tp * pp), kv_total / (tp * pp), ok, why)

    tp = 1
    while tp <= max_tp:
        if fits(tp, 1):
            return plan(tp, 1, True, f"tp{tp}: weights + KV fit one GPU group of {tp} within {budget:.0f} GB")
        tp *= 2
    tp = 1 << int(math.log2(max_tp))
    for pp in range(2, gpus // tp + 1):
        if fits(tp, pp):
            return plan(tp, pp, True, f"tp{tp} x pp{pp}: one NVLink domain is not enough")
    pp = max(1, gpus // tp)
    return plan(tp, pp, False, "does not fit: add GPUs, quantise the weights or shorten the KV budget")


def estimate_decode_tok_s(spec: ModelSpec, plan: Plan, batch: int, hbm_gbs: float = 6500.0,
                          efficiency: float = 0.5) -> float:
    """Bandwidth model of decode throughput: each step streams the weights and the KV once."""
    per_step_s = (plan.weight_gb_per_gpu + plan.kv_gb_per_gpu) * 1e9 / (hbm_gbs * 1e9 * efficiency)
    return plan.dp * batch / per_step_s if per_step_s > 0 else math.inf
