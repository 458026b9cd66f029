"""The end-to-end pipeline validator passes on the tiny model."""
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM
from openmini_v1_b200.validate import validate


def test_validator_tiny():
    r = validate(DecoderLM(tiny(), device="cpu", seed=0), max_model_len=128, steps=6)
    assert r["ok"], r
