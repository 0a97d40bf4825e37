"""Shared pytest configuration.

Tests marked ``gpu`` need a B200 (sm_100a) and the in-tree ``omnicoder._C``
extension; everything else runs on CPU (multi-rank tests use the ``gloo``
backend on 127.0.0.1).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100a device and the compiled extension")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def cuda_ext():
    """The compiled extension on a machine with a CUDA device; skips on CPU-only machines."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from omnicoder.ops import _ext

    return _ext.load()


@pytest.fixture(autouse=True)
def _check_device_status(request):
    """After every GPU test, the device status block must be clean."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from omnicoder.ops import _ext

    C = _ext.load()
    torch.cuda.synchronize()
    code, info, count = C.status()
    C.status_reset()
    assert code == 0, f"device status code {code} (info {info}, {count} errors)"
