import json
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "htn-2026_b200")
for p in (REPO, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_golden(name: str) -> dict:
    with open(os.path.join(GOLDEN, f"{name}.json")) as f:
        return json.load(f)


_STATES = {}


def synth_state(n_layers: int, seed: int = 0):
    """Seeded synthetic Qwen3 state dict (cached per process)."""
    from decode_b200 import synth

    key = (n_layers, seed)
    if key not in _STATES:
        cfg = synth.qwen3_config(n_layers)
        _STATES[key] = (synth.make_state_dict(cfg, seed), cfg)
    return _STATES[key]


@pytest.fixture(scope="session")
def golden_config0():
    return load_golden("config0")


@pytest.fixture(scope="session")
def golden_b3():
    return load_golden("b3_s17")
