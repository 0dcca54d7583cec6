"""Test configuration: the `gpu` marker, repo on sys.path, and shared fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def kb():
    """The klein_b200 package with its library loaded (fails loudly when the library is missing)."""
    import klein_b200

    klein_b200.lib()
    return klein_b200


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    return torch.device("cuda:0")
