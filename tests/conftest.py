"""Shared fixtures.  `-m "not gpu"` runs on CPU; `-m gpu` needs a B200."""
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tt-lab_b200" / "python"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


_LAYERS = {}


def synth_layer(seed, experts, layer=0, zipf_s=None, norm=False):
    """Cached host copy of one seeded synthetic layer."""
    from ttl_moe import synth
    key = (seed, experts, layer, zipf_s, norm)
    if key not in _LAYERS:
        _LAYERS[key] = synth.layer_host(seed, layer, experts, zipf_s=zipf_s, norm=norm)
    return _LAYERS[key]


@pytest.fixture(scope="session")
def layer32():
    return synth_layer(0, 32)


@pytest.fixture(scope="session")
def layer128():
    return synth_layer(1, 128)
