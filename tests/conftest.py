import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "causal-conv1d-cute_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(autouse=True)
def _device_checks(request):
    """GPU tests run with the kernels' index-check status word on and assert it stays clear."""
    if request.node.get_closest_marker("gpu") is None:
        yield
        return
    import causal_conv1d_cute as C

    C.set_device_checks(True)
    C.device_status()
    yield
    bad = C.device_status()
    assert bad == 0 or getattr(request.node, "_expect_status", False), f"device status {bad}"
