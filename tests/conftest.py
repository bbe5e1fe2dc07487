import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(ROOT / "tests" / "golden" / "golden.npz")


@pytest.fixture(autouse=True)
def _clean_device_errors(request):
    """Start every GPU test with no sticky device-error bits left by an
    earlier test (some tests record a bad label or a pipeline timeout on
    purpose; the library reports those bits at the next call)."""
    if request.node.get_closest_marker("gpu") is not None:
        import torch

        if torch.cuda.is_available():
            from greyhound_b200 import _lib

            torch.cuda.synchronize()
            _lib.take_device_errors(0)
    yield
