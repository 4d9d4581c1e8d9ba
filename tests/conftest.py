"""pytest configuration: the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs on machines without a GPU (CPU oracle, host runtime,
gloo multi-process tests); ``-m gpu`` needs a B200 and the built extension.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the sm_100a extension")
    config.addinivalue_line("markers", "slow: long-running test")
    config.addinivalue_line("markers", "multigpu: needs 2+ CUDA devices")


@pytest.fixture
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    return torch.device("cuda", 0)
