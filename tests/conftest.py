import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "sglang0.5.18-opt_b200")
for p in (REPO, PKG_ROOT, os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)


def _ensure_built():
    """Build the in-tree library once if it is missing (CPU tests load it; GPU tests call it)."""
    import glob

    pkg = os.path.join(PKG_ROOT, "hcu_ops")
    if os.path.exists(os.path.join(pkg, "libhcu_indexer.so")) and glob.glob(os.path.join(pkg, "_C*.so")):
        return
    import build  # sglang0.5.18-opt_b200/build.py

    build.build()


def pytest_configure(config):
    _ensure_built()
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: larger shapes")


@pytest.fixture(scope="session")
def dev():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def hcu(dev):
    """The product package; import failure (library not built) is a test failure, never a skip."""
    import hcu_ops

    hcu_ops.read_device_status(clear=True)
    return hcu_ops


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """Every GPU test must leave the library's device status word clear."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import hcu_ops

    st = hcu_ops.read_device_status(clear=True)
    allowed = getattr(request.node, "allowed_status", 0)
    assert st & ~allowed == 0, f"device status bits set: {st:#x}"
