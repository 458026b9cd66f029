"""The shipped config files load with the expected sections and values."""
import os

from openmini_v1_b200.config.settings import load_config

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shipped_configs_load():
    s = load_config(os.path.join(ROOT, "config", "server.toml"))
    assert s.server.port == 50051 and s.model.weight_format == "q4"
    m70 = load_config(os.path.join(ROOT, "config", "model_70b.toml"))
    assert m70.model.preset == "llama70b" and m70.distributed_inference.tp_degree == 8
    m14 = load_config(os.path.join(ROOT, "config", "model_14b.toml"))
    assert m14.model.preset == "dsa14b" and m14.engine.max_num_seqs == 16
