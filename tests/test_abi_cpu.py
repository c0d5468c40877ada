"""CPU-only checks of the C ABI library: it loads without a GPU driver, exports every
function that include/*.h declares, and reports (rather than crashes on) a missing device."""
import ctypes

import pytest

from c3_b200 import _lib


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _lib.declared_symbols()
    assert "c3cu_linear_bias_relu_fwd" in declared
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, f"declared in include/*.h but not exported: {missing}"


def test_version_and_status_calls_without_gpu():
    import torch
    lib = _lib.load()
    assert lib.c3cu_version() >= 1
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; the no-device path is not reachable")
    assert lib.c3cu_device_check() == -5  # C3CU_ERR_UNSUPPORTED
    assert "device" in _lib.last_error().lower()
    # entry points refuse cleanly before touching memory
    rc = lib.c3cu_linear_bias_relu_fwd(None, None, None, None, None, 1, 1, 1, 0, None)
    assert rc == -5


def test_workspace_size_queries_are_pure_host():
    lib = _lib.load()
    assert lib.c3cu_relu_mask_db_workspace(16384, 4096) >= 32 * 4096 * 4
    assert lib.c3cu_relu_mask_db_workspace(0, 10) > 0
    assert lib.c3cu_sum_rows_f32_workspace(5, 5) > 0


def test_device_wrapper_passes_host_calls_through():
    """on_tensor_device leaves calls without CUDA tensors alone (no device is touched)."""
    import torch
    from c3_b200 import _lib

    @_lib.on_tensor_device
    def f(a, b=None, xs=()):
        return a.sum() + (0 if b is None else b.sum()) + sum(x.sum() for x in xs)

    t = torch.ones(3)
    assert float(f(t, b=t, xs=[t, t])) == 12.0
