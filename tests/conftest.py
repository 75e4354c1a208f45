import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built CUDA extension")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def host():
    from gollek_b200.native import host_ext
    return host_ext()


@pytest.fixture(scope="session")
def tiny_cfg():
    from gollek_b200.config import preset
    return preset("tiny-llama")


@pytest.fixture(scope="session")
def tiny_weights(tiny_cfg):
    from gollek_b200.models.reference import init_random_weights
    return init_random_weights(tiny_cfg, seed=0)
