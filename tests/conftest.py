import os
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multi_gpu: needs >= 2 CUDA GPUs")
    config.addinivalue_line("markers", "distributed: spawns CPU/Gloo ranks")


def pytest_collection_modifyitems(config, items):
    has_gpu = torch.cuda.is_available()
    n = torch.cuda.device_count() if has_gpu else 0
    for item in items:
        if "gpu" in item.keywords and not has_gpu:
            item.add_marker(pytest.mark.skip(reason="no CUDA device"))
        if "multi_gpu" in item.keywords and n < 2:
            item.add_marker(pytest.mark.skip(reason="needs >= 2 CUDA GPUs"))


@pytest.fixture(scope="session")
def lib():
    from minitp_b200 import _lib
    from minitp_b200.build import build

    build()
    return _lib.load()


def golden(name: str):
    import numpy as np

    return np.load(os.path.join(GOLDEN, name))
