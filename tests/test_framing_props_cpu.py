"""Framing round trips (hypothesis) for the C++ runtime's wire formats: worker task /
result frames, and gateway frames fed to the incremental decoder in arbitrary chunk
sizes, decode to what was encoded; arbitrary bytes never crash the decoder (it
returns None, a frame, or raises ValueError)."""
from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200 import _native

rt = _native.rt()
sessions = st.text(alphabet=st.characters(min_codepoint=33, max_codepoint=126), max_size=36)
frames = st.lists(st.tuples(st.integers(0, 255), sessions, st.booleans(), st.binary(max_size=300)), min_size=1,
                  max_size=8)


@settings(max_examples=150, deadline=None)
@given(fs=frames, cuts=st.lists(st.integers(1, 64), min_size=1, max_size=40))
def test_gateway_frames_any_chunking(fs, cuts):
    wire = b"".join(rt.encode_gateway(t, s, st_, p) for t, s, st_, p in fs)
    d = rt.GatewayDecoder(1 << 20)
    got, i, k = [], 0, 0
    while i < len(wire):
        n = cuts[k % len(cuts)]
        d.feed(wire[i:i + n])
        i, k = i + n, k + 1
        while (x := d.next()) is not None:
            got.append(x)
    assert got == [(t, s.ljust(36), st_, p) for t, s, st_, p in fs]
    assert d.buffered() == 0


@settings(max_examples=150, deadline=None)
@given(tid=st.integers(0, 2 ** 64 - 1), ok=st.booleans(), data=st.binary(max_size=500))
def test_task_and_result_frames(tid, ok, data):
    assert rt.decode_task(rt.encode_task(tid, data)) == (tid, data)
    assert rt.decode_result(rt.encode_result(tid, ok, data)) == (tid, ok, data)


@settings(max_examples=200, deadline=None)
@given(junk=st.binary(max_size=200))
def test_decoder_survives_arbitrary_bytes(junk):
    d = rt.GatewayDecoder(64)
    d.feed(junk)
    for _ in range(8):
        try:
            x = d.next()
        except (ValueError, UnicodeDecodeError):
            break
        if x is None:
            break
        assert len(x) == 4 and isinstance(x[3], bytes)
