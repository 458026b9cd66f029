"""Control plane on CPU: router strategies, coordinator + worker processes with a
worker that dies mid-stream (heartbeat / connection failure -> its tasks fail over),
and the parallel-strategy planner."""
import multiprocessing as mp
import os
import time

from openmini_v1_b200.parallel.cluster import (PRESETS, Coordinator, ModelSpec, Router, estimate_decode_tok_s,
                                               plan_parallelism, run_worker)


def test_router_strategies():
    r = Router("round_robin")
    for n in "abc":
        r.add(n)
    assert [r.select() for _ in range(6)] == list("abcabc")
    w = Router("weighted")
    w.add("big", 3.0)
    w.add("small", 1.0)
    picks = [w.select() for _ in range(8)]
    assert picks.count("big") == 6 and picks.count("small") == 2
    ll = Router("least_loaded")
    ll.add("x")
    ll.add("y")
    assert {ll.select(), ll.select()} == {"x", "y"}
    ll.done("x", 0.01)
    assert ll.select() == "x"
    lat = Router("latency")
    lat.add("fast")
    lat.add("slow")
    lat.done(lat.select(), 0.0)
    lat.nodes["fast"].ewma_latency_s, lat.nodes["slow"].ewma_latency_s = 0.01, 1.0
    assert lat.select() == "fast"
    lat.mark("fast", False)
    assert lat.select() == "slow"


def _square(x):
    time.sleep(0.02)
    return x * x


def _worker(addr, name, die_after):
    if die_after is not None:
        n = {"k": 0}

        def h(x):
            n["k"] += 1
            if n["k"] > die_after:
                os._exit(1)  # the process dies with a task in flight
            return _square(x)
        run_worker(addr, name, h)
    else:
        run_worker(addr, name, _square)


def test_coordinator_failover():
    co = Coordinator(heartbeat_timeout_s=1.0, strategy="round_robin")
    ctx = mp.get_context("spawn")
    ps = [ctx.Process(target=_worker, args=(co.address, "w0", None)),
          ctx.Process(target=_worker, args=(co.address, "w1", 2))]
    for p in ps:
        p.start()
    try:
        assert co.wait_workers(2, 60)
        tids = [co.submit(i) for i in range(20)]
        res = co.collect(tids, timeout=60)
        assert [res[t]["result"] for t in tids] == [i * i for i in range(20)]
        assert any(e[0] == "dead" and e[1] == "w1" for e in co.events)
        assert co.router.nodes["w0"].completed >= 18
    finally:
        co.shutdown()
        for p in ps:
            p.join(10)
            if p.is_alive():
                p.kill()


def test_planner():
    spec7, _, _ = PRESETS["llama-7b"]
    p = plan_parallelism(spec7, gpus=8, kv_tokens=64 * 1280)
    assert p.fits and p.tp == 1 and p.dp == 8
    spec70, _, _ = PRESETS["llama-70b"]
    p70 = plan_parallelism(spec70, gpus=8)
    assert p70.fits and p70.tp >= 1 and p70.weight_gb_per_gpu + p70.kv_gb_per_gpu <= 162
    huge = ModelSpec(400.0, 120, 16384, 16, 128)
    ph = plan_parallelism(huge, gpus=16)
    assert ph.tp == 8 and ph.pp == 2 and ph.fits
    assert not plan_parallelism(huge, gpus=8).fits
    assert estimate_decode_tok_s(spec70, p70, batch=256) > 0
