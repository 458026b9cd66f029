"""ZeRO-style sharded AdamW on 2 gloo ranks equals unsharded torch AdamW on the
averaged gradient; optimizer memory per rank halves; memory estimator."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from openmini_v1_b200.train.zero import estimate_memory


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model(seed=0):
    torch.manual_seed(seed)
    return torch.nn.Sequential(torch.nn.Linear(7, 13), torch.nn.Tanh(), torch.nn.Linear(13, 3))


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from openmini_v1_b200.train.zero import ShardedAdamW
        m, ref = _model(), _model()
        opt = ShardedAdamW(m.parameters(), lr=1e-2, weight_decay=0.1)
        ropt = torch.optim.AdamW(ref.parameters(), lr=1e-2, weight_decay=0.1)
        g = torch.Generator().manual_seed(1)
        for step in range(5):
            xs = [torch.randn(8, 7, generator=g) for _ in range(world)]
            opt.zero_grad()
            m(xs[rank]).pow(2).mean().backward()
            opt.step()
            ropt.zero_grad()
            sum(ref(x).pow(2).mean() for x in xs).div(world).backward()
            ropt.step()
        err = max(float((a - b).abs().max()) for a, b in zip(m.parameters(), ref.parameters()))
        full = 3 * sum(p.numel() for p in ref.parameters()) * 4
        q.put((rank, err, opt.state_bytes(), full))
    finally:
        dist.destroy_process_group()


def test_sharded_adamw_matches_adamw():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(60)
    for rank, err, sb, full in res:
        assert err < 1e-5, (rank, err)
        assert sb <= full / 2 + 12


def test_memory_estimator():
    a = estimate_memory(7, dp=8, zero_stage=0)
    b = estimate_memory(7, dp=8, zero_stage=3)
    assert a.optimizer_gb == 84.0 and b.optimizer_gb == 10.5 and b.weights_gb == 14 / 8
    assert b.total_gb < a.total_gb
