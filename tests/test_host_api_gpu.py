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


def test_cfg1_training_loop_through_the_api(cuda_device):
    """The cfg1 MLP trained as a host framework drives C3 (tests/cpp/api_drive.cpp): after the
    hot-path threshold every hidden-layer region runs through RegionFusionRegistry::find ->
    executeFusedWithInputs, the backward nodes through C3BackwardCapture::tryExecuteBackward,
    and logits, loss and parameters stay bit-identical to the oracle's loop."""
    import json
    import subprocess

    from tests.cpp import build as cpp_build
    exe = cpp_build.build_drive()
    r = subprocess.run([str(exe), "mlp", "12"], capture_output=True, text=True, timeout=600)
    rec = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    assert r.returncode == 0, (rec, r.stderr[-2000:])
    t = rec["timed"]
    assert t["region_hits"] == 2 * 12 and t["region_misses"] == 0
    assert t["bw_hits"] >= 5 * 12  # 2 ReLU + 3 MatMul nodes per step (Add stays on the host)
    assert rec["logits_bit_exact"] and rec["loss_bit_exact"] and rec["params_bit_exact"]


def test_cfg2_region_through_the_api_with_host_tensors(cuda_device):
    """executeFusedWithInputs on host bf16 tensors (the drop-in contract: copies in, kernel,
    copies out), with B on the host and resident on the device: same bits both ways, and
    sampled rows within 2e-2 of the oracle."""
    import json
    import subprocess

    from tests.cpp import build as cpp_build
    exe = cpp_build.build_drive()
    r = subprocess.run([str(exe), "region", "1024", "512", "768", "2"], capture_output=True, text=True,
                       timeout=600)
    rec = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    assert r.returncode == 0, (rec, r.stderr[-2000:])
    assert rec["parity"]["same_bits_both_ways"] and rec["parity"]["max_rel"] <= 2e-2
