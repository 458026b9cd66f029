"""Collectives on real process groups (gloo, 2 CPU ranks) and the in-process
LocalComm fake; tensor-parallel decoder math equals the single-rank model."""
import os
import socket
import threading

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from openmini_v1_b200.parallel.comm import CollectiveOps, LocalComm, ReduceOp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = CollectiveOps()
        t = torch.full((4,), float(rank + 1))
        c.all_reduce(t)
        g = c.all_gather(torch.tensor([rank, rank]), dim=0)
        rs = c.reduce_scatter(torch.arange(4, dtype=torch.float32) * (rank + 1))
        b = c.broadcast(torch.tensor([rank * 10]), root=1)
        mx = c.all_reduce(torch.tensor([float(rank)]), ReduceOp.MAX)
        # tensor-parallel decoder vs single-rank
        from openmini_v1_b200.models.config import tiny
        from openmini_v1_b200.models.llama import DecoderLM, ForwardBatch
        from openmini_v1_b200.parallel.state import ParallelState
        par = ParallelState.build(tp=world)
        cfg = tiny()
        full = DecoderLM(cfg, device="cpu", seed=0)
        shard = DecoderLM(cfg, par=par, device="cpu", materialize=False)
        shard.set_comm(CollectiveOps(par.tp_group))
        _shard_weights(full, shard, par.tp_rank, world)
        T = 9
        i32 = dict(dtype=torch.int32)
        toks = torch.arange(100, 100 + T, dtype=torch.int32)
        outs = []
        for m in (full, shard):
            kv = m.allocate_kv(2)
            fb = ForwardBatch(toks, torch.arange(T, **i32), torch.arange(T, **i32), torch.arange(2, **i32)[None],
                              torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T, torch.tensor([T - 1]))
            outs.append(m.logits(m(fb, kv)))
        # sequence-parallel transport (token-sharded residual, fused reduce/norm/gather events)
        from openmini_v1_b200.parallel.symm import make_sp
        shard.set_sp(make_sp(par, "cpu", 64, cfg.hidden_size, dtype=torch.float32))
        kv = shard.allocate_kv(2)
        fb = ForwardBatch(toks, torch.arange(T, **i32), torch.arange(T, **i32), torch.arange(2, **i32)[None],
                          torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T, torch.tensor([T - 1]))
        sp_out = shard.logits(shard(fb, kv))
        q.put((rank, t.tolist(), g.tolist(), rs.tolist(), b.tolist(), mx.tolist(),
               float((outs[0] - outs[1]).abs().max()), float((outs[0] - sp_out).abs().max())))
    finally:
        dist.destroy_process_group()


def _shard_weights(full, shard, r, tp):
    hq, hkv, hd, F = shard.hq, shard.hkv, shard.hd, shard.ffn
    shard.embed, shard.norm = full.embed, full.norm
    V = full.cfg.vocab_size // tp
    shard.lm_head = full.lm_head[r * V:(r + 1) * V]
    shard.layers = []
    for L in full.layers:
        Hq, Hkv = full.hq, full.hkv
        q = L["qkv"][: Hq * hd].view(Hq, hd, -1)[r * hq:(r + 1) * hq].reshape(hq * hd, -1)
        k = L["qkv"][Hq * hd:(Hq + Hkv) * hd].view(Hkv, hd, -1)[r * hkv:(r + 1) * hkv].reshape(hkv * hd, -1)
        v = L["qkv"][(Hq + Hkv) * hd:].view(Hkv, hd, -1)[r * hkv:(r + 1) * hkv].reshape(hkv * hd, -1)
        Ff = full.ffn
        g = L["gate_up"][:Ff][r * F:(r + 1) * F]
        u = L["gate_up"][Ff:][r * F:(r + 1) * F]
        shard.layers.append({
            "attn_norm": L["attn_norm"], "ffn_norm": L["ffn_norm"],
            "qkv": torch.cat([q, k, v]).contiguous(),
            "o": L["o"][:, r * hq * hd:(r + 1) * hq * hd].contiguous(),
            "gate_up": torch.cat([g, u]).contiguous(),
            "down": L["down"][:, r * F:(r + 1) * F].contiguous(),
        })


def test_gloo_collectives_and_tp_decoder():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for rank, t, g, rs, b, mx, tp_err, sp_err in res:
        assert t == [3.0] * 4
        assert g == [0, 0, 1, 1]
        assert rs == ([0.0, 3.0] if rank == 0 else [6.0, 9.0])
        assert b == [10]
        assert mx == [1.0]
        assert tp_err < 1e-4, tp_err
        assert sp_err < 1e-4, sp_err


def test_local_comm_threads():
    comms = LocalComm.create(3)
    out = [None] * 3

    def run(r):
        t = torch.tensor([float(r)])
        comms[r].all_reduce(t)
        g = comms[r].all_gather(torch.tensor([r]), dim=0)
        rs = comms[r].reduce_scatter(torch.ones(6) * (r + 1))
        out[r] = (t.item(), g.tolist(), rs.tolist())

    th = [threading.Thread(target=run, args=(r,)) for r in range(3)]
    for t in th:
        t.start()
    for t in th:
        t.join(30)
    for r in range(3):
        assert out[r][0] == 3.0 and out[r][1] == [0, 1, 2] and out[r][2] == [6.0, 6.0]


def test_backend_registry_and_failover():
    import threading
    import torch
    from openmini_v1_b200.parallel.comm import FailoverComm, LocalComm, make_backend

    class Broken:
        def all_reduce(self, t, op=None):
            raise RuntimeError("NCCL watchdog: link down")

    comms = LocalComm.create(2)
    assert isinstance(make_backend("local", rank=0, shared=comms[0].shared), LocalComm)
    events, out = [], [None, None]

    def run(r):
        fc = FailoverComm(Broken(), comms[r], on_failover=lambda n, e: events.append((r, n)),
                          names=("nccl", "local"))
        out[r] = (fc.all_reduce(torch.full((3,), float(r + 1))), fc.backend_name, list(fc.failures))
    ts = [threading.Thread(target=run, args=(r,)) for r in range(2)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(10)
    for r in range(2):
        val, name, fails = out[r]
        assert torch.equal(val, torch.full((3,), 3.0)) and name == "local" and fails[0][0] == "all_reduce"
    assert sorted(events) == [(0, "local"), (1, "local")]
    import pytest
    with pytest.raises(KeyError):
        make_backend("carrier-pigeon")
