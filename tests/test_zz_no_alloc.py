"""The allocation-free backward pre-pass, c3cu_relu_mask_db_noalloc, called through the C ABI.

It serves callers that cannot allocate device memory themselves (a host framework whose
allocator owns all device memory, or a latency-critical path that must not let cudaMalloc
synchronise the device): its scratch is a fixed array inside the library. This test checks
it against the workspace-taking entry point, c3cu_relu_mask_db, on two calls in a row (the
second call reuses the array with the first call's contents still in it), and that sizes
beyond the array are refused. The file name sorts last so that a run stopping at the first
failure has already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

from c3_b200 import _lib

pytestmark = pytest.mark.gpu

_vp, _i64 = ctypes.c_void_p, ctypes.c_int64


def _abi():
    L = _lib.load()
    L.c3cu_relu_mask_db_noalloc.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _vp]
    L.c3cu_relu_mask_db_noalloc.restype = ctypes.c_int
    L.c3cu_relu_mask_db.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _vp, ctypes.c_size_t, _vp]
    L.c3cu_relu_mask_db.restype = ctypes.c_int
    L.c3cu_relu_mask_db_workspace.argtypes = [_i64, _i64]
    L.c3cu_relu_mask_db_workspace.restype = ctypes.c_size_t
    return L


def _case(M, N, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    dY = (torch.randn((M, N), generator=g, device=dev) * 1e-3).to(torch.bfloat16)
    words = (N + 31) // 32
    mask = torch.randint(-2**31, 2**31 - 1, (M, words), generator=g, device=dev, dtype=torch.int64)
    return dY, mask.to(torch.int32)


def _with_workspace(L, dY, mask, stream):
    M, N = dY.shape
    dZ = torch.empty_like(dY)
    db = torch.empty(N, dtype=torch.float32, device=dY.device)
    nb = L.c3cu_relu_mask_db_workspace(M, N)
    ws = torch.empty(nb, dtype=torch.uint8, device=dY.device)
    rc = L.c3cu_relu_mask_db(dY.data_ptr(), mask.data_ptr(), dZ.data_ptr(), db.data_ptr(), M, N,
                             ws.data_ptr(), nb, stream)
    assert rc == 0, _lib.last_error()
    return dZ, db


def _no_alloc(L, dY, mask, stream):
    M, N = dY.shape
    dZ = torch.empty_like(dY)
    db = torch.empty(N, dtype=torch.float32, device=dY.device)
    rc = L.c3cu_relu_mask_db_noalloc(dY.data_ptr(), mask.data_ptr(), dZ.data_ptr(), db.data_ptr(), M, N,
                                     stream)
    assert rc == 0, _lib.last_error()
    return dZ, db


# cfg3's shape, a ragged shape, and the largest size the 4 MiB array holds at N = 4096
@pytest.mark.parametrize("M,N", [(16384, 4096), (1000, 300), (130560, 4096)])
def test_no_alloc_matches_workspace_entry_point_twice(cuda_device, M, N):
    L = _abi()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    # Two different inputs in a row: the second call must not see the first call's state.
    for seed in (1, 2):
        dY, mask = _case(M, N, seed, cuda_device)
        dZ_ref, db_ref = _with_workspace(L, dY, mask, stream)
        dZ, db = _no_alloc(L, dY, mask, stream)
        torch.cuda.synchronize()
        # dZ is a masked copy: identical bits; db within the pre-pass tolerance of the other
        # tests (1e-5 of the column's sum of magnitudes)
        assert torch.equal(dZ.view(torch.int16), dZ_ref.view(torch.int16))
        bound = 1e-5 * dZ_ref.float().abs().sum(0) + 1e-12
        assert bool(((db - db_ref).abs() <= bound).all())


def test_no_alloc_empty_batch_writes_zero_db(cuda_device):
    """M = 0 is an empty reduction: every column of db is +0, whatever db held before."""
    L = _abi()
    N = 300
    db = torch.full((N,), float("nan"), dtype=torch.float32, device=cuda_device)
    dummy = torch.empty(16, dtype=torch.uint8, device=cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    rc = L.c3cu_relu_mask_db_noalloc(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), db.data_ptr(),
                                     0, N, stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert bool((db == 0).all()) and not bool(torch.signbit(db).any())


def test_no_alloc_refuses_sizes_beyond_its_array(cuda_device):
    L = _abi()
    M, N = 130561, 4096  # one row more than the 4 MiB array holds at N = 4096
    assert L.c3cu_relu_mask_db_workspace(M - 1, N) <= 4 * 1024 * 1024
    assert L.c3cu_relu_mask_db_workspace(M, N) > 4 * 1024 * 1024
    rc = L.c3cu_relu_mask_db_noalloc(None, None, None, None, M, N, None)
    assert rc == -6  # C3CU_ERR_WORKSPACE, refused before anything is launched
    assert "scratch" in _lib.last_error()
