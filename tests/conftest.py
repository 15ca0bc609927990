import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="CUDA GPU not available")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    assert torch.cuda.is_available(), "GPU tests need CUDA"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"built for sm_100a, found sm_{major}{minor}"
    return torch.device("cuda", 0)


@pytest.fixture(scope="session", autouse=True)
def _lib_built():
    """Make sure the in-tree library exists (builds it with nvcc when stale)."""
    if os.environ.get("DU_SKIP_BUILD") == "1":
        return
    from dominusultra_b200 import build

    build.build()
