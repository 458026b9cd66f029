"""In-process collectives (``LocalComm``, the N-rank fake the tensor-parallel unit
tests run on) against direct torch reductions (hypothesis): every reduce op,
broadcast from any root, all-gather along a dimension and reduce-scatter, for
random world sizes and shapes, with the ranks running as threads."""
import threading

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200.parallel.comm import LocalComm, ReduceOp


def _run(W, fn):
    comms = LocalComm.create(W)
    out = [None] * W
    errs = []

    def go(r):
        try:
            out[r] = fn(r, comms[r])
        except Exception as e:  # report instead of hanging the other ranks' joins
            errs.append(e)
    th = [threading.Thread(target=go, args=(r,)) for r in range(W)]
    for t in th:
        t.start()
    for t in th:
        t.join(30)
    assert not errs, errs
    return out


@settings(max_examples=40, deadline=None)
@given(W=st.integers(1, 5), n=st.integers(1, 6), seed=st.integers(0, 10 ** 6),
       op=st.sampled_from(list(ReduceOp)), root=st.integers(0, 4))
def test_local_collectives(W, n, seed, op, root):
    g = torch.Generator().manual_seed(seed)
    xs = [torch.randn(W * n, 3, generator=g) for _ in range(W)]
    stack = torch.stack(xs)
    want = {ReduceOp.SUM: stack.sum(0), ReduceOp.AVG: stack.mean(0), ReduceOp.MAX: stack.max(0).values,
            ReduceOp.MIN: stack.min(0).values, ReduceOp.PROD: stack.prod(0)}[op]
    root %= W

    def fn(r, c):
        t = xs[r].clone()
        c.all_reduce(t, op)
        b = xs[r].clone()
        c.broadcast(b, root)
        ag = c.all_gather(xs[r][:n], dim=1)
        rs = c.reduce_scatter(xs[r], dim=0)
        return t, b, ag, rs
    for r, (t, b, ag, rs) in enumerate(_run(W, fn)):
        assert torch.allclose(t, want, rtol=1e-5, atol=1e-5)
        assert torch.equal(b, xs[root])
        assert torch.equal(ag, torch.cat([x[:n] for x in xs], dim=1))
        assert torch.allclose(rs, stack.sum(0)[r * n:(r + 1) * n], atol=1e-5)
