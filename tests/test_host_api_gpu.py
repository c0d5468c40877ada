"""Runs the GPU cases of the C++ host-API tests: the C3 registry / engine / backward-capture
API driving the sm_100a kernels, checked against the oracle (fp32 path bit-exact, bf16
tensor-core path within 2e-2)."""
import subprocess

import pytest

from tests.cpp.build import build

pytestmark = pytest.mark.gpu


def test_host_api_gpu(cuda_device):
    exe = build()
    r = subprocess.run([str(exe), "--gpu"], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout
