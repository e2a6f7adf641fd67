import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on CPU")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    # A gpu-marked test on a machine without a GPU is skipped, never silently passed.
    if cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device on this machine")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
