import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; parity against the oracle")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device in this environment")
    import c3_b200
    c3_b200.device_check()  # raises C3CUError when the device is not sm_100
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _no_fault_after_gpu_test(request):
    """Every GPU test ends by reading the kernels' fault word (bounded waits that gave up)."""
    yield
    if request.node.get_closest_marker("gpu") is not None:
        import torch
        if torch.cuda.is_available():
            import c3_b200
            assert c3_b200.fault_status() == 0
