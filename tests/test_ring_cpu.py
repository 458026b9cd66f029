"""Ring attention (context parallelism) on 3 gloo CPU ranks equals full causal
attention over the whole sequence; the LSE merge is exact."""
import math
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from openmini_v1_b200.parallel.ring_attention import _attend_cpu, merge


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(T=60, H=4, Hkv=2, D=16):
    g = torch.Generator().manual_seed(0)
    return (torch.randn(T, H, D, generator=g), torch.randn(T, Hkv, D, generator=g),
            torch.randn(T, Hkv, D, generator=g))


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from openmini_v1_b200.parallel.ring_attention import ring_attention
        Q, K, V = _data()
        C = Q.shape[0] // world
        sl = slice(rank * C, (rank + 1) * C)
        out, lse = ring_attention(Q[sl], K[sl], V[sl])
        want, wlse = _attend_cpu(Q, K, V, 1 / math.sqrt(16), causal=True)
        q.put((rank, float((out - want[sl]).abs().max()), float((lse - wlse[sl]).abs().max())))
    finally:
        dist.destroy_process_group()


def test_merge_is_exact():
    Q, K, V = _data()
    o, l = _attend_cpu(Q, K, V, 0.25, causal=False)
    o1, l1 = _attend_cpu(Q, K[:25], V[:25], 0.25, causal=False)
    o2, l2 = _attend_cpu(Q, K[25:], V[25:], 0.25, causal=False)
    om, lm = merge(o1, l1, o2, l2)
    assert torch.allclose(om, o, atol=1e-5) and torch.allclose(lm, l, atol=1e-5)


def test_ring_attention_three_ranks():
    world, port = 3, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(60)
    for rank, e_out, e_lse in res:
        assert e_out < 1e-5 and e_lse < 1e-5, (rank, e_out, e_lse)
