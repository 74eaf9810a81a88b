import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
# the reference's trained checkpoints, staged (not committed) by __graft_entry__.build()
STAGED_WEIGHTS = ROOT / "oracle" / "_ref" / "weights"
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def staged(name):
    path = STAGED_WEIGHTS / name
    if not path.exists():
        pytest.skip(f"reference checkpoint {name} is not staged in oracle/_ref/weights")
    return path


@pytest.fixture(scope="session")
def cuda_available():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
