import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _no_device_timeouts(request):
    """After every GPU test: no bounded device wait may have timed out."""
    yield
    if "gpu" not in request.keywords:
        return
    import ctypes

    import torch
    if not torch.cuda.is_available():
        return
    from zerollm_b200 import lib
    torch.cuda.synchronize()
    code = ctypes.c_int(0)
    lib.load().zl_device_error(ctypes.byref(code))
    assert code.value == 0, f"device-side bounded wait timed out (code {code.value})"
