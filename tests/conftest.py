import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly (never skip) when run with -m gpu on a box without
    # the library; on CPU runs they are deselected by the marker expression.
    pass


@pytest.fixture(scope="session")
def golden():
    import torch
    return torch.load(ROOT / "tests" / "golden" / "moe_golden.pt", weights_only=True)
