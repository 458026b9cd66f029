"""Pipeline parallelism (p2p send/recv, microbatched) and expert parallelism
(all-to-all dispatch / combine) on 2 gloo CPU ranks give the single-rank
model's logits."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _batch(T, nblocks=2):
    from openmini_v1_b200.models.llama import ForwardBatch
    i32 = dict(dtype=torch.int32)
    toks = torch.arange(100, 100 + T, dtype=torch.int32)
    return ForwardBatch(toks, torch.arange(T, **i32), torch.arange(T, **i32), torch.arange(nblocks, **i32)[None],
                        torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T, torch.tensor([3, T - 1]))


def _pp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from openmini_v1_b200.models.config import tiny
        from openmini_v1_b200.models.llama import DecoderLM
        from openmini_v1_b200.parallel.pipeline import PipelineStage, stage_layers
        from openmini_v1_b200.parallel.state import ParallelState
        cfg = tiny()
        cfg.num_layers = 3
        par = ParallelState.build(pp=world)
        full = DecoderLM(cfg, device="cpu", seed=1)
        T = 11
        want = full.logits(full(_batch(T), full.allocate_kv(2)))
        stage = PipelineStage.from_model(full, par, world, par.pp_rank)
        res = {}
        for mb in (1, 3):
            out = stage.forward(_batch(T), stage.allocate_kv(2), microbatches=mb)
            lg = stage.logits(out)
            tok = torch.zeros(2, dtype=torch.int64)
            if stage.last:
                tok = lg.argmax(-1)
                res[mb] = float((lg - want).abs().max())
            stage.broadcast_tokens(tok)
            res[f"tok{mb}"] = tok.tolist() == want.argmax(-1).tolist()
        q.put((rank, res, stage_layers(3, world, par.pp_rank)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _ep_worker(rank, world, port, q, capacity=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from openmini_v1_b200.models.config import tiny
        from openmini_v1_b200.models.llama import DecoderLM
        from openmini_v1_b200.parallel.expert import ExpertParallel
        from openmini_v1_b200.parallel.state import ParallelState
        cfg = tiny()
        cfg.moe.num_experts, cfg.moe.top_k, cfg.moe.expert_ffn = 4, 2, 64
        full = DecoderLM(cfg, device="cpu", seed=2)
        T = 13 + rank * 4  # ranks hold different token counts
        fb = _batch(T)
        fb.record_routing = {}
        want = full.logits(full(fb, full.allocate_kv(2)))
        par = ParallelState.build(ep=world)
        m = DecoderLM(cfg, device="cpu", seed=2)
        ep = ExpertParallel(par.ep_group, capacity_factor=capacity, max_tokens=32 if capacity else None)
        m.set_ep(ep, par.ep_rank)
        assert len(m.layers[0]["experts_gate_up"]) == 4 // world
        fb2 = _batch(T)
        fb2.record_routing = {}
        got = m.logits(m(fb2, m.allocate_kv(2)))
        same_routing = all(torch.equal(fb.record_routing[i], fb2.record_routing[i]) for i in fb.record_routing)
        dropped = int(ep.dropped) if ep.dropped is not None else 0
        q.put((rank, float((got - want).abs().max()), same_routing, dropped))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(target, world=2):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    return res


def test_pipeline_parallel_matches_single_rank():
    res = _run(_pp_worker)
    assert [r[2] for r in res] == [(0, 2), (2, 3)]
    last = res[-1][1]
    assert last[1] < 1e-4 and last[3] < 1e-4, last
    assert all(r[1]["tok1"] and r[1]["tok3"] for r in res)


def test_expert_parallel_matches_single_rank():
    for rank, err, same, _ in _run(_ep_worker):
        assert same
        assert err < 1e-4, (rank, err)


def _ep_fixed_big(rank, world, port, q):
    _ep_worker(rank, world, port, q, capacity=2.0)


def _ep_fixed_small(rank, world, port, q):
    _ep_worker(rank, world, port, q, capacity=0.25)


def test_expert_parallel_fixed_capacity():
    """Equal-split dispatch without host synchronisation: with room for every pair the
    result equals one rank's; with a small capacity pairs are dropped and counted."""
    for rank, err, same, dropped in _run(_ep_fixed_big):
        assert same and dropped == 0 and err < 1e-4, (rank, err, dropped)
    res = _run(_ep_fixed_small)
    assert sum(r[3] for r in res) > 0


def _tp_sample_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from openmini_v1_b200 import ops
        from openmini_v1_b200.models.config import tiny
        from openmini_v1_b200.models.llama import DecoderLM
        from openmini_v1_b200.parallel.comm import CollectiveOps
        from openmini_v1_b200.parallel.state import ParallelState
        cfg = tiny()
        par = ParallelState.build(tp=world)
        m = DecoderLM(cfg, par=par, device="cpu", seed=3)
        m.set_comm(CollectiveOps(par.tp_group))
        assert m.vocab_local * world == cfg.vocab_size  # the vocabulary-sharded head
        res = []
        for B in (5, 8):  # 5: padded to a multiple of the TP size
            g = torch.Generator().manual_seed(B)
            x = torch.randn(B, cfg.hidden_size, generator=g)
            temp = torch.rand(B, generator=g) + 0.3
            temp[0] = 0.0  # one greedy row
            top_p = torch.rand(B, generator=g) * 0.5 + 0.5
            top_k = torch.tensor([0, 5] * B, dtype=torch.int32)[:B]
            rng = torch.randint(0, 1 << 30, (B, 2), generator=g)
            want_t, want_lp, _ = ops.sample(m.logits(x), temp, top_p, top_k, rng)
            got_t, got_lp, _ = m.sample(x, temp, top_p, top_k, rng)
            res.append((got_t.tolist() == want_t.tolist(), float((got_lp - want_lp).abs().max())))
        q.put((rank, res))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_tp_row_parallel_sampling_matches_gathered_logits():
    """Row-parallel sampling under TP (all-to-all of vocab shards, each rank samples its
    rows, all-gather of tokens) draws exactly what sampling the gathered logits draws."""
    world = 2
    q = mp.get_context("spawn").Queue()
    procs = [mp.get_context("spawn").Process(target=_tp_sample_worker, args=(r, world, _free_port_shared(), q))
             for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, res in out:
        for same, lp_err in res:
            assert same and lp_err < 1e-5, (rank, res)


_PORT = None


def _free_port_shared():
    global _PORT
    if _PORT is None:
        _PORT = _free_port()
    return _PORT
