"""Sampler oracle properties (hypothesis) on random logits: the kept set of
temperature -> top-k -> top-p always holds the most likely token, has at most k
members, covers at least p of the probability mass and is a prefix of the tokens
ordered by logit (ties kept together); the drawn token is in the kept set; greedy
rows take the argmax; a draw depends only on (seed, offset)."""
import math

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200.ops import reference as ref


@settings(max_examples=150, deadline=None)
@given(seed=st.integers(0, 2 ** 31 - 1), V=st.integers(2, 300), t=st.floats(0.05, 3.0),
       k=st.integers(0, 50), p=st.floats(0.05, 1.0))
def test_cutoff_and_draw(seed, V, t, k, p):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(1, V, generator=g) * 3
    x = logits[0] / t
    x = x - x.max()
    keep = ref._cutoff_mask(x, k, p)
    prob = torch.softmax(x, 0)
    assert keep[int(torch.argmax(x))]
    if 0 < k < V:
        # ties at the k-th value may keep a few more
        assert int(keep.sum()) <= k + int((x == torch.topk(x, k).values[-1]).sum()) - 1
    if p < 1.0:
        mass = float(prob[keep].sum())
        zk = float(prob[ref._cutoff_mask(x, k, 1.0)].sum())
        assert mass >= p * zk - 1e-5
    lo = float(x[keep].min())
    assert bool((x[~keep] < lo).all()) if (~keep).any() else True      # a prefix by logit
    rng = torch.tensor([[seed, 7]])
    tok, lp, mask = ref.sample(logits, torch.tensor([t]), torch.tensor([p]), torch.tensor([k]), rng)
    assert bool(mask[0, int(tok[0])]) and bool(keep[int(tok[0])])
    assert math.isclose(float(lp[0]), float(torch.log_softmax(x, 0)[int(tok[0])]), rel_tol=1e-4, abs_tol=1e-4)
    tok2, _, _ = ref.sample(torch.cat([torch.randn(1, V), logits]), torch.tensor([1.0, t]), torch.tensor([1.0, p]),
                            torch.tensor([0, k]), torch.tensor([[1, 1], [seed, 7]]))
    assert int(tok2[1]) == int(tok[0])                                  # independent of the batch row
    g0, _, _ = ref.sample(logits, torch.tensor([0.0]), torch.tensor([p]), torch.tensor([k]), rng)
    assert int(g0[0]) == int(torch.argmax(logits[0]))
