import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "mamba-cpu_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size configuration (seconds of oracle time)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _no_device_fault(request):
    """GPU tests: no kernel may have recorded a fault (a bounded wait that gave up)."""
    yield
    if "gpu" in request.keywords:
        import torch

        if torch.cuda.is_available():
            from mamba_cpu_b200 import _lib

            assert _lib.device_fault() == 0, "a kernel recorded a device-side fault"
