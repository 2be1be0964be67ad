import os
import sys
from pathlib import Path

# every pipelined kernel launched by the tests reads back its status word
os.environ.setdefault("GPA_CHECK_STATUS", "1")

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import torch

    def load(name):
        return torch.load(GOLDEN / name, weights_only=False)
    return load
