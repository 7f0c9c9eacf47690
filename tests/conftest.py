import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_ROOT = ROOT / "breeze-tts-2_b200"
for p in (str(ROOT), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    """Loader for the committed golden fixtures (tests/golden/*.npz)."""
    cache = {}

    def load(name: str):
        if name not in cache:
            cache[name] = np.load(GOLDEN / name)
        return cache[name]

    return load


def has_cuda() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False


@pytest.fixture(scope="session")
def lib():
    """The product C-ABI library, loaded through the package's loader."""
    from breeze_b200 import _lib

    return _lib.load()


@pytest.fixture(autouse=True)
def _require_gpu_for_gpu_tests(request):
    if request.node.get_closest_marker("gpu") and not has_cuda():
        if os.environ.get("BQ_REQUIRE_GPU"):
            pytest.fail("GPU test run without a CUDA device")
        pytest.skip("needs a CUDA device")
