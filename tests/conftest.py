import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")


@pytest.fixture(scope="session")
def orc():
    """The CPU oracle (test infrastructure, oracle/)."""
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device; GPU tests fail (not skip) when it is missing."""
    import torch

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    import rsllm_b200  # noqa: F401  (loads the CUDA library or raises)

    return torch.device("cuda", 0)
