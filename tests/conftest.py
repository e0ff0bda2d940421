import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


@pytest.fixture(scope="session")
def native():
    from polylora_b200 import _native

    return _native


@pytest.fixture()
def cuda_status_clean(native):
    """Asserts the kernels raised no device status bits during the test."""
    native.device_status(clear=True)
    yield
    status = native.device_status(clear=True)
    assert status == 0, f"device status raised: {status:#x}"


os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")
