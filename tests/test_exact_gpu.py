"""The fp32 path reproduces the reference's arithmetic bit for bit (max_diff = 0, the
reference's own parity claim for MatMul/Add): sequential-k fmul/fadd GEMM, the region's
T + b then maxnum, and the row-ordered SumReduce."""
import numpy as np
import pytest
import torch

import oracle
from c3_b200 import exact
from tests.helpers import unpack_mask

pytestmark = pytest.mark.gpu

SHAPES = [(128, 784, 256), (128, 256, 128), (128, 128, 10), (1, 1, 1), (65, 33, 17), (300, 1000, 70)]


def _rand(shape, seed, lo=-1.0, hi=1.0):
    return (torch.rand(shape, generator=torch.Generator().manual_seed(seed)) * (hi - lo) + lo).float()


@pytest.mark.parametrize("M,K,N", SHAPES)
@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
def test_matmul_bit_exact(cuda_device, M, K, N, ta, tb):
    A = _rand((K, M) if ta else (M, K), M + K)
    B = _rand((N, K) if tb else (K, N), K + N)
    out = exact.matmul(A.to(cuda_device), B.to(cuda_device), ta, tb).cpu().numpy()
    ref = oracle.matmul(A.numpy(), B.numpy(), transA=ta, transB=tb)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_matmul_bias_init_and_act(cuda_device, act):
    M, K, N = 64, 96, 48
    A, B, bias = _rand((M, K), 1), _rand((K, N), 2), _rand((N,), 3)
    out = exact.matmul(A.to(cuda_device), B.to(cuda_device), bias=bias.to(cuda_device), act=act).cpu().numpy()
    ref = oracle.matmul(A.numpy(), B.numpy(), bias=bias.numpy(), act=act)
    if act in (0, 1):
        assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
    else:  # expf / tanhf come from different libms: a few ulp
        assert np.abs(out - ref).max() <= 4e-7 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_region_forward_bit_exact(cuda_device, M, K, N):
    X, B, b = _rand((M, K), 10, 0, 1), _rand((K, N), 11, -0.1, 0.1), _rand((N,), 12, -0.1, 0.1)
    out, z, mask = exact.region_forward(X.to(cuda_device), B.to(cuda_device), b.to(cuda_device), want_z=True)
    ref, zref = oracle.region_fwd(X.numpy(), B.numpy(), b.numpy())
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(z.cpu().numpy().view(np.uint32), zref.view(np.uint32))
    assert np.array_equal(unpack_mask(mask.cpu().numpy().view(np.uint32), N), zref > 0)


def test_region_forward_scalar_bias_broadcast(cuda_device):
    X, B, b = _rand((33, 20), 20), _rand((20, 12), 21), _rand((1,), 22)
    out, _, _ = exact.region_forward(X.to(cuda_device), B.to(cuda_device), b.to(cuda_device))
    ref, _ = oracle.region_fwd(X.numpy(), B.numpy(), b.numpy())
    assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("M,N", [(128, 256), (16384, 10), (1, 7), (1000, 1000)])
def test_sum_rows_bit_exact(cuda_device, M, N):
    x = _rand((M, N), M * 7 + N)
    out = exact.sum_rows(x.to(cuda_device)).cpu().numpy()
    ref = oracle.sum_reduce(x.numpy(), 0)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_exact_kernels_reproduce_golden_vectors(cuda_device):
    """The GPU fp32 path against the golden vectors of the independent restatement."""
    import json
    from pathlib import Path
    gold = json.loads((Path(__file__).resolve().parent / "golden" / "golden.json").read_text())
    arr = lambda v, s=None: (np.array(v, np.uint32).view(np.float32).reshape(s) if s else
                             np.array(v, np.uint32).view(np.float32))
    c = gold["region_fwd"]
    M, K, N = c["M"], c["K"], c["N"]
    out, z, _ = exact.region_forward(torch.from_numpy(arr(c["X"], (M, K))).to(cuda_device),
                                     torch.from_numpy(arr(c["B"], (K, N))).to(cuda_device),
                                     torch.from_numpy(arr(c["b"])).to(cuda_device), want_z=True)
    assert np.array_equal(out.cpu().numpy().view(np.uint32).ravel(), np.array(c["out"], np.uint32))
    assert np.array_equal(z.cpu().numpy().view(np.uint32).ravel(), np.array(c["z"], np.uint32))
    for ta in (0, 1):
        for tb in (0, 1):
            c = gold[f"matmul_ta{ta}_tb{tb}"]
            A = torch.from_numpy(arr(c["A"], (K, M) if ta else (M, K))).to(cuda_device)
            B = torch.from_numpy(arr(c["B"], (N, K) if tb else (K, N))).to(cuda_device)
            got = exact.matmul(A, B, bool(ta), bool(tb)).cpu().numpy().view(np.uint32).ravel()
            assert np.array_equal(got, np.array(c["out"], np.uint32))


@pytest.mark.parametrize("M,K,N", [(128, 10, 128), (128, 128, 256), (77, 33, 65)])
def test_matmul_relu_bwd_bit_exact(cuda_device, M, K, N):
    """MatMul backward dA (grad @ W^T, W stored [N, K]) fused with the upstream ReLU backward:
    the same bits as the oracle's matmul followed by Mul(Gt(z, 0), .)."""
    G, W, z = _rand((M, K), 30), _rand((N, K), 31), _rand((M, N), 32)
    out = exact.matmul_relu_bwd(G.to(cuda_device), W.to(cuda_device), z.to(cuda_device), trans_b=True)
    da = oracle.matmul(G.numpy(), W.numpy(), transB=True)
    ref = oracle.relu_bwd(da, z.numpy())
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("M,K,N", [(256, 128, 128), (784, 128, 256), (128, 128, 10), (5, 0, 7)])
def test_matmul_colsum_bit_exact(cuda_device, M, K, N):
    """MatMul backward dB (A^T @ grad, A stored [K, M]) and the Add backward's SumReduce of the
    same grad from one launch: both bit-identical to the oracle's separate kernels."""
    A, G = _rand((K, M), 40), _rand((K, N), 41)
    dW, db = exact.matmul_colsum(A.to(cuda_device), G.to(cuda_device), trans_a=True)
    ref_w = oracle.matmul(A.numpy(), G.numpy(), transA=True) if K > 0 else np.zeros((M, N), np.float32)
    ref_b = oracle.sum_reduce(G.numpy(), 0) if K > 0 else np.zeros(N, np.float32)
    assert np.array_equal(dW.cpu().numpy().view(np.uint32), ref_w.view(np.uint32))
    assert np.array_equal(db.cpu().numpy().view(np.uint32), ref_b.view(np.uint32))
