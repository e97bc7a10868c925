"""Test configuration: the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs everywhere (oracle against the golden vectors, host logic, the C-ABI
library's exports); ``-m gpu`` needs a B200 and calls the kernels through the C ABI.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100a device (B200)")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    # A gpu test on a machine without a GPU is an error, not a skip, unless it was deselected.
    pass


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"the kernels are built for sm_100a, this device is sm_{major}{minor}")
    return torch.device("cuda:0")
