"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on any machine (oracle pins, host logic, library
loading); `-m gpu` runs the parity tests proper on a B200.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "paged-kv-cache_b200"))
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a CUDA device")
    return torch.device("cuda:0")
