import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(autouse=True)
def _no_device_error(request):
    """Every GPU test must leave the kernels' bounded-wait error word at zero."""
    yield
    if "gpu" in request.keywords:
        import torch
        if torch.cuda.is_available():
            from flashgmm_b200 import _lib
            code = _lib.load().fgmm_device_error(1)
            assert code == 0, f"a tensor-core kernel recorded wait-timeout code {code}"
