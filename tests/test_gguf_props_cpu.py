"""GGUF writer -> C++ parser round trip (hypothesis): metadata of every value type
(bool, 32/64-bit integers, float32, UTF-8 strings, homogeneous arrays) and F32 / F16
tensors of random shapes come back unchanged, with the data section aligned."""
import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200.gguf.constants import GGMLType
from openmini_v1_b200.gguf.reader import GGUFReader
from openmini_v1_b200.gguf.writer import GGUFWriter

f32 = st.floats(width=32, allow_nan=False, allow_infinity=False)
text = st.text(alphabet=st.characters(blacklist_categories=("Cs",)), max_size=30)
scalar = st.one_of(st.booleans(), st.integers(-2 ** 63, 2 ** 64 - 1), f32, text)
array = st.one_of(st.lists(st.integers(0, 2 ** 32 - 1), max_size=20), st.lists(f32, min_size=1, max_size=20),
                  st.lists(text, min_size=1, max_size=10), st.lists(st.booleans(), min_size=1, max_size=10),
                  st.lists(st.integers(-2 ** 31, -1), min_size=1, max_size=10))
meta = st.dictionaries(st.from_regex(r"[a-z][a-z0-9_.]{0,20}", fullmatch=True), st.one_of(scalar, array), max_size=12)
shapes = st.lists(st.integers(1, 9), min_size=1, max_size=3)


@settings(max_examples=60, deadline=None)
@given(md=meta, shps=st.lists(shapes, max_size=4), seed=st.integers(0, 1000))
def test_gguf_round_trip(tmp_path_factory, md, shps, seed):
    md = {k: v for k, v in md.items() if not k.startswith("general.")}
    path = str(tmp_path_factory.mktemp("g") / "t.gguf")
    w = GGUFWriter(path, "llama")
    for k, v in md.items():
        w.add_kv(k, v)
    rng = np.random.default_rng(seed)
    arrs = []
    for i, shp in enumerate(shps):
        a = rng.standard_normal(shp).astype(np.float32)
        typ = GGMLType.F32 if i % 2 == 0 else GGMLType.F16
        w.add_tensor(f"t{i}", a, typ)
        arrs.append((a, typ))
    w.write()
    r = GGUFReader(path)
    for k, v in md.items():
        got = r.metadata[k]
        if isinstance(v, float):
            assert got == float(np.float32(v))
        elif isinstance(v, list) and v and isinstance(v[0], float):
            assert list(got) == [float(np.float32(x)) for x in v]
        else:
            assert (list(got) if isinstance(v, list) else got) == v, (k, v, got)
    assert r.data_offset % int(r.metadata.get("general.alignment", 32)) == 0
    for i, (a, typ) in enumerate(arrs):
        t = r.tensors[f"t{i}"]
        assert t.shape == a.shape and t.type == typ
        want = a if typ == GGMLType.F32 else a.astype(np.float16).astype(np.float32)
        assert np.array_equal(t.to_numpy(), want)
