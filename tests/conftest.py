import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    # A GPU test that runs without a GPU must fail loudly (there is no CPU
    # fallback), so the gpu marker is never auto-skipped here; the driver
    # selects with -m gpu / -m "not gpu".
    return None


@pytest.fixture(scope="session")
def golden_dir():
    return REPO / "tests" / "golden"


def cuda_available():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


os.environ.setdefault("PYTHONHASHSEED", "0")
