"""Property test of the C++ paged-KV block manager (hypothesis-driven random
operation sequences): a sequence's block table always covers its tokens, no block
is owned by two sequences unless shared by fork or the prefix cache (reference
counts equal the number of tables holding the block), ``append_need`` /
``can_append`` predict exactly whether an append succeeds, copy-on-write gives the
writer a private last block, and freeing every sequence returns every block."""
import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from openmini_v1_b200 import _native

BS = 16


def _check(bm, live):
    owners = {}
    for sid, toks in live.items():
        bt = list(bm.block_table(sid))
        assert len(bt) == (len(toks) + BS - 1) // BS, (sid, len(bt), len(toks))
        assert bm.seq_len(sid) == len(toks)
        for b in bt:
            owners[b] = owners.get(b, 0) + 1
    for b, n in owners.items():
        assert bm.ref_count(b) == n, (b, bm.ref_count(b), n)
    assert bm.num_free() + len(owners) <= bm.num_blocks


ops = st.lists(st.tuples(st.sampled_from(["alloc", "append", "fork", "free"]), st.integers(0, 7),
                         st.integers(1, 40), st.integers(0, 3)), min_size=1, max_size=60)


@pytest.mark.parametrize("prefix", [True, False])
@settings(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(seq=ops)
def test_block_manager_invariants(prefix, seq):
    bm = _native.rt().BlockManager(24, BS, prefix)
    live = {}
    prompts = [[7] * 40, [7] * 20 + [8] * 20, [9] * 33, [1, 2, 3] * 11]   # shared prefixes for the cache
    for op, sid, n, which in seq:
        if op == "alloc" and sid not in live:
            toks = prompts[which][:n]
            if bm.can_allocate(len(toks)):
                bm.allocate(sid, toks)
                live[sid] = list(toks)
            else:
                with pytest.raises(RuntimeError):
                    bm.allocate(sid, toks)
        elif op == "append" and sid in live:
            toks = [100 + sid] * (n % 20 + 1)
            need = bm.append_need(sid, len(toks))
            assert bm.can_append(sid, len(toks)) == (need <= bm.num_free())
            if need <= bm.num_free():
                before = list(bm.block_table(sid))
                cow = bm.append(sid, toks)
                live[sid] += toks
                after = list(bm.block_table(sid))
                for src, dst in cow:      # the writer's partial block was replaced by a private copy
                    assert src in before and dst in after and src not in after and bm.ref_count(dst) == 1
            else:
                with pytest.raises(RuntimeError):
                    bm.append(sid, toks)
        elif op == "fork" and sid in live:
            child = 100 + which * 10 + sid
            if child not in live:
                bm.fork(sid, child)
                live[child] = list(live[sid])
        elif op == "free" and sid in live:
            bm.free(sid)
            del live[sid]
        _check(bm, live)
    for sid in list(live):
        bm.free(sid)
    assert bm.num_free() == bm.num_blocks
