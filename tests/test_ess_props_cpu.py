"""Two-tier elastic storage (hypothesis over random put / get / remove sequences and
every eviction policy): neither tier ever holds more than its budget, a key is in at
most one tier, and ``get`` returns exactly the tensor last stored under the key or
None once it has been dropped -- never another key's data."""
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200.engine.ess import ElasticStorage

ops = st.lists(st.tuples(st.sampled_from(["put", "get", "remove"]), st.integers(0, 12), st.integers(1, 70)),
               min_size=1, max_size=80)


@pytest.mark.parametrize("policy", ["lru", "lfu", "adaptive"])
@settings(max_examples=60, deadline=None)
@given(seq=ops)
def test_tiers_budgets_and_contents(policy, seq):
    s = ElasticStorage(device_budget_bytes=64 * 4, host_budget_bytes=160 * 4, policy=policy)
    last = {}
    for op, key, n in seq:
        if op == "put":
            t = torch.full((n,), float(key * 1000 + n))
            if 4 * n > s.host_budget:
                with pytest.raises(ValueError):
                    s.put(key, t)
                continue
            s.put(key, t)
            last[key] = t
        elif op == "get":
            got = s.get(key)
            if got is not None:
                assert key in last and torch.equal(got.cpu(), last[key])
        else:
            s.remove(key)
            last.pop(key, None)
        assert s.dev_used() <= s.dev_budget and s.host_used() <= s.host_budget
        assert not (set(s.dev) & set(s.host))
        for k in list(s.dev) + list(s.host):
            assert k in last
