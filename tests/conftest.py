import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def headline_case():
    """The 128K headline layer (seed 1000, 256 mixture
    components, nprobe 384) for the CPU restatement, built once per session."""
    from tests.helpers import Case

    return Case(context=131072, nprobe=384, seed=1000, components=256)
