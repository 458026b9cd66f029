"""Dynamic strategy adjuster (bottleneck detection, guarded switch, rollback) and
UDP discovery between two local nodes (join, update, leave)."""
import socket
import time

from openmini_v1_b200.parallel.adjuster import (AdjusterConfig, Discovery, DynamicAdjuster, PeerInfo,
                                                PerformanceMetrics)
from openmini_v1_b200.parallel.cluster import PRESETS


def _m(tps, p99=100.0, comm=0.05, mem=0.5):
    return PerformanceMetrics(p50_ms=p99 / 2, p99_ms=p99, throughput_tps=tps, comm_frac=comm, mem_util=mem)


def test_adjuster_switch_cooldown_and_rollback():
    t = [0.0]
    spec = PRESETS["llama-70b"][0]
    adj = DynamicAdjuster(spec, gpus=8, batch=64, cfg=AdjusterConfig(min_samples=3, cooldown_s=10, min_gain=0.05),
                          clock=lambda: t[0])
    start = (adj.current.tp, adj.current.pp)
    assert adj.evaluate().action == "keep"  # not enough samples
    for _ in range(3):
        adj.record(_m(1000))
    d = adj.evaluate()
    assert d.action == "keep" and d.bottleneck == "none"
    for _ in range(3):
        adj.record(_m(1000, comm=0.4))
    d = adj.evaluate()
    assert d.bottleneck == "communication"
    assert d.action == "switch"  # a layout with less TP communication is predicted to be better
    assert (d.plan.tp, d.plan.pp) != start
    for _ in range(3):
        adj.record(_m(500, comm=0.1))  # worse after the switch
    t[0] += 1
    r = adj.evaluate()
    assert r.action == "rollback" and (adj.current.tp, adj.current.pp) == start
    for _ in range(3):
        adj.record(_m(1000, comm=0.4))
    assert adj.evaluate().reason == "cooldown"
    assert all(c.fits for c in adj.candidates())


def _free_port():
    s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_discovery_join_update_leave():
    pa, pb = _free_port(), _free_port()
    a = Discovery(PeerInfo("a", "10.0.0.1:9000", 8, 180.0), pa, peers=[("127.0.0.1", pb)], timeout_s=0.6).start()
    b = Discovery(PeerInfo("b", "10.0.0.2:9000", 4, 180.0), pb, peers=[("127.0.0.1", pa)], timeout_s=0.6).start()
    try:
        deadline = time.time() + 5
        while time.time() < deadline and not (a.alive() and b.alive()):
            time.sleep(0.05)
        assert [p.node_id for p in a.alive()] == ["b"] and a.total_gpus() == 12
        b.info.gpus = 8
        deadline = time.time() + 5
        while time.time() < deadline and ("updated", "b") not in a.events:
            time.sleep(0.05)
        assert ("updated", "b") in a.events and a.total_gpus() == 16
        b.stop()
        deadline = time.time() + 5
        while time.time() < deadline and ("left", "b") not in a.events:
            time.sleep(0.05)
        assert ("left", "b") in a.events and a.alive() == []
    finally:
        a.stop()
