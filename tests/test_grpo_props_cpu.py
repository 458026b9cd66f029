"""GRPO objective properties (hypothesis): group-relative advantages have zero mean
and unit population scale per group (all-zero for a constant group); the K3 KL
estimate is non-negative, zero exactly at equal log-probs and unbiased for KL(p||ref)
in expectation over p; the PPO-clip loss equals -A r inside the trust region and is
flat in r outside it on the side the advantage favours."""
import math

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200.rl.grpo import group_relative_advantage, k3_kl, ppo_clip_loss


@settings(max_examples=80, deadline=None)
@given(G=st.integers(2, 16), n=st.integers(1, 5), seed=st.integers(0, 10 ** 6), const=st.booleans())
def test_advantages(G, n, seed, const):
    g = torch.Generator().manual_seed(seed)
    r = torch.ones(n * G, dtype=torch.float64) if const else torch.randn(n * G, generator=g, dtype=torch.float64)
    a = group_relative_advantage(r, G).view(n, G)
    assert torch.allclose(a.mean(1), torch.zeros(n, dtype=a.dtype), atol=1e-9)
    if const:
        assert bool((a == 0).all())
    else:
        var = r.view(n, G).var(1, unbiased=False)
        assert torch.allclose((a ** 2).mean(1), var / (var + 1e-8), atol=1e-9)  # 1 unless var ~ eps


@settings(max_examples=80, deadline=None)
@given(seed=st.integers(0, 10 ** 6))
def test_k3_kl(seed):
    g = torch.Generator().manual_seed(seed)
    lp = torch.randn(50, generator=g, dtype=torch.float64)
    rp = lp + torch.randn(50, generator=g, dtype=torch.float64) * 0.5
    assert float(k3_kl(lp, rp)) >= 0 and float(k3_kl(lp, lp)) == 0.0
    # unbiased: E_{x~p}[k3] = KL(p || ref) for categorical p, ref
    V = 6
    p = torch.softmax(torch.randn(V, generator=g, dtype=torch.float64), 0)
    q = torch.softmax(torch.randn(V, generator=g, dtype=torch.float64), 0)
    d = q.log() - p.log()
    expect_k3 = float((p * (torch.exp(d) - 1 - d)).sum())
    kl = float((p * (p.log() - q.log())).sum())
    assert abs(expect_k3 - kl) < 1e-9


@settings(max_examples=80, deadline=None)
@given(lr=st.floats(-0.5, 0.5), adv=st.floats(-3, 3).filter(lambda x: abs(x) > 1e-3), eps=st.floats(0.05, 0.4))
def test_ppo_clip(lr, adv, eps):
    logp = torch.tensor([lr], dtype=torch.float64, requires_grad=True)
    old = torch.zeros(1, dtype=torch.float64)
    A = torch.tensor([adv], dtype=torch.float64)
    loss = ppo_clip_loss(logp, old, A, clip_eps=eps)
    r = math.exp(lr)
    loss.backward()
    if 1 - eps < r < 1 + eps:
        assert abs(float(loss.detach()) + adv * r) < 1e-9
        assert float(logp.grad) != 0.0
    elif (adv > 0 and r > 1 + eps) or (adv < 0 and r < 1 - eps):
        assert float(logp.grad) == 0.0            # clipped: no push further out of the region
    else:
        assert abs(float(loss.detach()) + adv * r) < 1e-9  # the pessimistic unclipped term
