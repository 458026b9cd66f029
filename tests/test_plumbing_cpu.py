"""Host plumbing on CPU: thread pool, partitioners, per-core actors and router,
connection pool, memory / load monitors, device arena, two-tier elastic storage."""
import threading
import time

import pytest
import torch

from openmini_v1_b200.engine.ess import ElasticStorage, StridePrefetcher
from openmini_v1_b200.hardware.memory import (CRITICAL, NORMAL, WARNING, DeviceArena, LoadMonitor,
                                              MemoryMonitor, MemorySnapshot, kv_block_budget)
from openmini_v1_b200.serve.concurrency import (ConnectionPool, CoreRouter, DynamicScheduler, GuidedScheduler,
                                                PoolConfig, TaskPartitioner, ThreadPool, spawn_core_actors)


def test_thread_pool_priority_results_and_errors():
    pool = ThreadPool(PoolConfig(size=1))
    gate = threading.Event()
    order = []
    pool.execute(gate.wait)  # occupies the only worker
    time.sleep(0.05)
    hs = [pool.execute(order.append, i) for i in range(3)]
    hh = pool.execute_high_priority(order.append, "hi")
    gate.set()
    assert pool.wait_completion(5)
    assert order == ["hi", 0, 1, 2]
    assert all(h.done() for h in hs + [hh])
    bad = pool.execute(lambda: 1 / 0)
    with pytest.raises(ZeroDivisionError):
        bad.result(5)
    assert pool.map(lambda x: x * x, range(5)) == [0, 1, 4, 9, 16]
    pool.shutdown()
    with pytest.raises(RuntimeError):
        pool.execute(print)
    assert PoolConfig.io_intensive().resolved_size() >= PoolConfig.compute_intensive().resolved_size()


def test_partitioners_cover_the_range_once():
    p = TaskPartitioner(workers=4, min_chunk=10)
    parts = p.partition_range(103)
    assert parts[0][0] == 0 and parts[-1][1] == 103 and len(parts) == 4
    assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
    assert TaskPartitioner(workers=8, min_chunk=100).optimal_parallelism(250) == 2
    for sched in (DynamicScheduler(97, 10), GuidedScheduler(97, 4, 3)):
        seen = []
        while (c := sched.next_chunk()) is not None:
            seen.extend(range(*c))
        assert seen == list(range(97))
    g = GuidedScheduler(100, 4, 2)
    sizes = []
    while (c := g.next_chunk()) is not None:
        sizes.append(c[1] - c[0])
    assert sizes[0] == 25 and sizes == sorted(sizes, reverse=True)


def test_core_actors_and_router():
    actors = spawn_core_actors(lambda x: x * 2, cores=[0, 0, 0], pin=False)
    try:
        for strat in ("round_robin", "least_connections", "consistent_hash"):
            r = CoreRouter(actors, strat)
            assert r.call(21, "s1").result == 42
        r = CoreRouter(actors, "round_robin")
        assert [r.select("") for _ in range(4)] == [0, 1, 2, 0]
        ch = CoreRouter(actors, "consistent_hash")
        assert len({ch.select("session-7") for _ in range(10)}) == 1  # sticky
        picks = {ch.select(f"s{i}") for i in range(200)}
        assert picks == {0, 1, 2}
        err = CoreRouter([spawn_core_actors(lambda x: 1 / 0, cores=[0], pin=False)[0]]).call(1)
        assert not err.ok and "ZeroDivisionError" in err.error
    finally:
        for a in actors:
            a.stop()


def test_connection_pool_reuse_bound_and_broken():
    made = []

    class Conn:
        def __init__(self):
            self.alive = True
            made.append(self)

        def close(self):
            self.alive = False

    pool = ConnectionPool(Conn, max_size=2, check=lambda c: c.alive)
    a = pool.acquire()
    b = pool.acquire()
    with pytest.raises(TimeoutError):
        pool.acquire(timeout=0.05)
    pool.release(a)
    assert pool.acquire() is a and pool.stats()["reused"] == 1
    pool.release(a)
    pool.release(b, broken=True)
    assert not b.alive
    with pool.connection() as c:
        assert c is a
    a.alive = False  # fails its health check: replaced
    c2 = pool.acquire()
    assert c2 is not a and len(made) == 3
    pool.release(c2)
    pool.close()


def test_memory_monitor_levels_and_budget():
    seq = iter([MemorySnapshot(100, 50), MemorySnapshot(100, 10, 1000, 100), MemorySnapshot(100, 2),
                MemorySnapshot(100, 60)])
    mon = MemoryMonitor(sampler=lambda: next(seq))
    seen = []
    mon.on_change(lambda lvl, s: seen.append(lvl))
    for _ in range(4):
        mon.poll()
    assert seen == [WARNING, CRITICAL, NORMAL]
    real = MemoryMonitor().poll()
    assert real.host_total > 0
    assert kv_block_budget(150 << 30, 180 << 30, 1 << 20, 0.9, 4 << 30) == (150 - 18 - 4) * 1024


def test_device_arena():
    ar = DeviceArena(4096)
    a = ar.alloc((3, 5), torch.float32)
    m = ar.mark()
    b = ar.alloc(100, torch.bfloat16)
    assert a.shape == (3, 5) and b.shape == (100,)
    assert (b.data_ptr() - a.data_ptr()) % 256 == 0
    ar.release_to(m)
    c = ar.alloc(100, torch.bfloat16)
    assert c.data_ptr() == b.data_ptr()
    with pytest.raises(MemoryError):
        ar.alloc(10000, torch.float32)
    ar.reset()
    assert ar.used == 0 and ar.peak > 0


class _FakeNVML:
    class U:
        gpu = 97

    def nvmlDeviceGetCount(self):
        return 2

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetUtilizationRates(self, h):
        return self.U()

    def nvmlDeviceGetTemperature(self, h, s):
        return 60 + 30 * h

    def nvmlDeviceGetPowerUsage(self, h):
        return 700000

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return 0x4 | (0x40 if h else 0)


def test_load_monitor_fake_nvml():
    mon = LoadMonitor(nvml=_FakeNVML())
    s = mon.sample()
    assert s.gpu_util == [97, 97] and s.gpu_temp_c == [60, 90] and s.gpu_power_w == [700.0, 700.0]
    assert s.gpu_throttle[0] == ["sw_power_cap"] and "hw_thermal_slowdown" in s.gpu_throttle[1]
    assert mon.overloaded(s)


@pytest.mark.parametrize("policy", ["lru", "lfu", "adaptive"])
def test_elastic_storage_tiers(policy):
    one = 4 * 256  # bytes of a [256] fp32 segment
    ess = ElasticStorage(device_budget_bytes=2 * one, host_budget_bytes=3 * one, policy=policy, prefetch=False)
    for i in range(4):
        ess.put(i, torch.full((256,), float(i)))
    assert ess.dev_used() <= 2 * one and ess.host_used() <= 3 * one
    assert sorted(k for k in range(4) if ess.tier(k) == "device") == [2, 3]
    assert ess.stats.demotions == 2
    t = ess.get(0)  # host hit -> promoted, someone demoted
    assert torch.equal(t, torch.zeros(256)) and ess.tier(0) == "device" and ess.stats.host_hits == 1
    for i in range(4, 8):
        ess.put(i, torch.full((256,), float(i)))
    assert ess.stats.drops >= 1 and ess.get(99) is None and ess.stats.misses == 1
    present = [k for k in range(8) if ess.tier(k)]
    for k in present:
        assert float(ess.get(k)[0]) == k


def test_lfu_keeps_hot_entry_and_prefetch():
    one = 4 * 256
    ess = ElasticStorage(2 * one, 8 * one, policy="lfu", prefetch=False)
    ess.put("hot", torch.ones(256))
    for _ in range(5):
        ess.get("hot")
    for i in range(3):
        ess.put(f"cold{i}", torch.zeros(256))
    assert ess.tier("hot") == "device"
    p = StridePrefetcher(depth=2)
    assert p.access(10) == [] and p.access(12) == [] and p.access(14) == [16, 18]
    assert p.pattern() == "strided"
    ess = ElasticStorage(2 * one, 16 * one, policy="lru", prefetch=True)
    for i in range(8):
        ess.put(i, torch.full((256,), float(i)))
    for i in (0, 1, 2):
        ess.get(i)
    assert ess.stats.prefetches >= 1 and ess.tier(3) == "device"
