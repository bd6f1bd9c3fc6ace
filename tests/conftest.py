import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden_v1.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


def _cuda_ok() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def native():
    """Builds (if stale) and loads the native library."""
    from dscquant_b200 import _lib, build

    build.build()
    return _lib.load()


@pytest.fixture(scope="session")
def oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc  # noqa: E402

    orc.build()
    return orc


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test: no kernel of the library raised its sticky status (an expired bounded
    wait or bad launch geometry), which would otherwise leave partial outputs unnoticed."""
    yield
    if "gpu" in request.keywords and _cuda_ok():
        from dscquant_b200 import ops

        assert ops.device_status(0) == 0, "a kernel raised the device status word during this test"


@pytest.fixture(scope="session")
def cuda_device(native):
    import torch

    torch.cuda.init()
    return torch.device("cuda", 0)
