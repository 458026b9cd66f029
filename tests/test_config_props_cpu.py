"""Server configuration round trip (hypothesis): any settings written with
``ServerConfig.to_toml`` read back (``from_str``) to an equal configuration,
including strings that need escaping and unknown keys kept in ``extra``."""
import dataclasses
import tomllib

from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200.config.settings import ServerConfig

text = st.text(alphabet=st.characters(blacklist_categories=("Cs",)), max_size=20)


def _mutate(cfg, draw_vals):
    for sec in dataclasses.fields(cfg):
        if sec.name == "extra":
            continue
        obj = getattr(cfg, sec.name)
        for f in dataclasses.fields(obj):
            cur = getattr(obj, f.name)
            v = draw_vals(type(cur))
            if v is not None:
                setattr(obj, f.name, v)


@settings(max_examples=60, deadline=None)
@given(data=st.data())
def test_toml_round_trip(data):
    cfg = ServerConfig()

    def draw(t):
        if not data.draw(st.booleans()):
            return None
        if t is bool:
            return data.draw(st.booleans())
        if t is int:
            return data.draw(st.integers(-2 ** 62, 2 ** 62))
        if t is float:
            return data.draw(st.floats(allow_nan=False, allow_infinity=False))
        if t is str:
            return data.draw(text)
        if t is list:
            return data.draw(st.lists(st.integers(0, 100), max_size=4))
        return None
    _mutate(cfg, draw)
    cfg.extra = data.draw(st.dictionaries(st.from_regex(r"[a-z][a-z0-9_]{0,8}", fullmatch=True),
                                          st.one_of(st.integers(0, 10), text), max_size=3))
    cfg.extra = {k: v for k, v in cfg.extra.items() if k not in {f.name for f in dataclasses.fields(cfg)}}
    t = cfg.to_toml()
    tomllib.loads(t)                      # valid TOML
    assert ServerConfig.from_str(t) == cfg
