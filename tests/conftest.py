"""Shared test configuration: the `gpu` marker and import paths."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run on the B200 box with -m gpu)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA GPU")
    import fast_forced_aligner_b200 as ffa
    ffa.load_extension()
    return torch.device("cuda", 0)
