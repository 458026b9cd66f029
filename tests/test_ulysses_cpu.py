"""Ulysses sequence parallelism (head / sequence all-to-all) on 2 gloo CPU ranks
equals full causal attention over the whole sequence, with grouped-query heads."""
import math
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from openmini_v1_b200.parallel.ring_attention import _attend_cpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(T=48, H=8, Hkv=2, D=16):
    g = torch.Generator().manual_seed(1)
    return (torch.randn(T, H, D, generator=g), torch.randn(T, Hkv, D, generator=g),
            torch.randn(T, Hkv, D, generator=g))


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from openmini_v1_b200.parallel.ulysses import ulysses_attention
        Q, K, V = _data()
        C = Q.shape[0] // world
        sl = slice(rank * C, (rank + 1) * C)
        out = ulysses_attention(Q[sl], K[sl], V[sl])
        want, _ = _attend_cpu(Q, K, V, 1 / math.sqrt(16), causal=True)
        full = ulysses_attention(Q[sl], K[sl], V[sl], causal=False)
        wfull, _ = _attend_cpu(Q, K, V, 1 / math.sqrt(16), causal=False)
        err = max(float((out - want[sl]).abs().max()), float((full - wfull[sl]).abs().max()))
        try:
            ulysses_attention(Q[sl, :3], K[sl], V[sl])
            bad = False
        except ValueError:
            bad = True
        q.put((rank, err, bad))
    except BaseException as e:
        q.put((rank, float("inf"), repr(e)))
    finally:
        dist.destroy_process_group()


def test_ulysses_two_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(60)
    for rank, err, bad in res:
        assert err < 1e-5 and bad is True, (rank, err, bad)
