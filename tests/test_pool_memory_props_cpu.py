"""Stateful properties (hypothesis) of the connection pool and the short-term memory
window: the pool never has more than max_size connections alive, never hands one
connection to two holders, reuses released ones and closes broken or failing ones;
the memory window stays within its token budget (keeping at least the last turn)
and always ends with the newest turn."""
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200.memory.dmn import ShortTermMemory
from openmini_v1_b200.serve.concurrency import ConnectionPool


class _Conn:
    n = 0

    def __init__(self):
        _Conn.n += 1
        self.id, self.closed, self.healthy = _Conn.n, False, True

    def close(self):
        self.closed = True


@settings(max_examples=80, deadline=None)
@given(ops=st.lists(st.tuples(st.sampled_from(["acq", "rel", "broken", "sick"]), st.integers(0, 9)), max_size=60),
       size=st.integers(1, 4))
def test_connection_pool(ops, size):
    pool = ConnectionPool(_Conn, max_size=size, check=lambda c: c.healthy)
    held, made = [], []
    for op, i in ops:
        if op == "acq":
            if len(held) == size:
                with pytest.raises(TimeoutError):
                    pool.acquire(timeout=0)
                continue
            c = pool.acquire(timeout=0)
            assert not c.closed and c not in held
            held.append(c)
            if c not in made:
                made.append(c)
        elif held:
            c = held.pop(i % len(held))
            if op == "sick":
                c.healthy = False            # fails the check when next taken from the idle list
            pool.release(c, broken=op == "broken")
            if op == "broken":
                assert c.closed
        alive = [c for c in made if not c.closed]
        assert len(alive) <= size and len(held) <= size
    for c in held:
        pool.release(c)
    again = [pool.acquire(timeout=0) for _ in range(size)]   # everything came back: a full pool again
    assert len({id(c) for c in again}) == size and all(not c.closed and c.healthy for c in again)


@settings(max_examples=80, deadline=None)
@given(turns=st.lists(st.text(alphabet="ab ", max_size=40), min_size=1, max_size=30), budget=st.integers(1, 30))
def test_short_term_window(turns, budget):
    m = ShortTermMemory(token_budget=budget)
    for i, t in enumerate(turns):
        m.add("s", "user" if i % 2 == 0 else "assistant", t)
        w = m.window("s")
        assert w and w[-1].text == t
        if len(w) > 1:
            assert sum(x.tokens for x in w) <= budget
    m.clear("s")
    assert m.window("s") == []
