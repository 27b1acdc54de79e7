import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture
def kernel_ok():
    """Fails the test if any kernel hit a bounded-wait limit while it ran."""
    from rs_nanogpt_b200.ops._ext import kernel_status
    kernel_status(True)
    yield
    import torch
    torch.cuda.synchronize()
    assert kernel_status(True) == 0, "a kernel hit its bounded-wait limit"
