import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

try:  # property tests draw the same examples on every run (set HYPOTHESIS_RANDOM=1 to explore)
    from hypothesis import settings as _hsettings
    _hsettings.register_profile("repeatable", derandomize=True, database=None)
    _hsettings.register_profile("explore")
    _hsettings.load_profile("explore" if os.environ.get("HYPOTHESIS_RANDOM") else "repeatable")
except ImportError:
    pass


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
