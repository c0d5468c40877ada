"""Bit-exact fp32 kernels (CUDA cores) restating the reference's fp32 loops: the c3.matmul
sequential-k reduction (src/C3/C3DialectLowering.cpp:467-610), the MatMul+Add+ReLU region
(src/C3/MLIRKernelGen.cpp:610-768), SumReduce axis 0 (src/C3/C3DialectLowering.cpp:382-465), and
two pairs of the captured backward fused into one launch each (MatMul dA + the upstream ReLU
backward; MatMul dB + the Add backward's SumReduce, src/C3/C3BackwardCapture.cpp:501-723)."""
from __future__ import annotations

import torch

from . import _lib
from .linear import _p, _require, _stream


def _f32(t, name, ndim: int = 2, shape=None):
    _require(t, name, torch.float32, ndim, shape)


def _bias(b, name: str):
    """Bias of the fp32 kernels: any contiguous fp32 vector of at least one element (read as
    bias[j] or bias[idx % numel], the reference's broadcast)."""
    _f32(b, name, 1)
    if b.numel() < 1:
        raise _lib.C3CUError(-1, name, "a bias needs at least one element")


def matmul(A: torch.Tensor, B: torch.Tensor, trans_a: bool = False, trans_b: bool = False,
           bias: torch.Tensor | None = None, act: int = 0) -> torch.Tensor:
    """out = act(bias_init + sum_k a(i,k) b(k,j)); A [M,K] ([K,M] if trans_a), B [K,N] ([N,K] if trans_b)."""
    _f32(A, "A")
    _f32(B, "B")
    M, K = (A.shape[1], A.shape[0]) if trans_a else (A.shape[0], A.shape[1])
    N = B.shape[0] if trans_b else B.shape[1]
    _f32(B, "B", 2, (N, K) if trans_b else (K, N))
    if bias is not None:
        _bias(bias, "bias")
        if bias.numel() not in (1, N):
            raise _lib.C3CUError(-1, "bias", f"a matmul bias holds 1 or N={N} elements, got {bias.numel()}")
    out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    rc = _lib.load().c3cu_matmul_f32(_p(A), _p(B), _p(out), M, K, N, int(trans_a), int(trans_b), _p(bias),
                                     0 if bias is None else bias.numel(), act, _stream(A.device))
    _lib.check(rc, "c3cu_matmul_f32")
    return out


def region_forward(X: torch.Tensor, B: torch.Tensor, b: torch.Tensor, trans_b: bool = False,
                   want_z: bool = False):
    """(out, z, mask) of the fp32 region: z = X B + b[idx % numel(b)], out = max(z, 0)."""
    _f32(X, "X")
    _f32(B, "B")
    _bias(b, "b")
    M, K = X.shape
    N = B.shape[0] if trans_b else B.shape[1]
    _f32(B, "B", 2, (N, K) if trans_b else (K, N))
    out = torch.empty((M, N), dtype=torch.float32, device=X.device)
    z = torch.empty_like(out) if want_z else None
    mask = torch.empty((M, (N + 31) // 32), dtype=torch.int32, device=X.device)
    rc = _lib.load().c3cu_region_fwd_f32(_p(X), _p(B), _p(b), b.numel(), _p(out), _p(z), _p(mask), M, K, N,
                                         int(trans_b), _stream(X.device))
    _lib.check(rc, "c3cu_region_fwd_f32")
    return out, z, mask


def sum_rows(x: torch.Tensor) -> torch.Tensor:
    _f32(x, "x")
    M, N = x.shape
    out = torch.empty(N, dtype=torch.float32, device=x.device)
    rc = _lib.load().c3cu_sum_rows_f32_exact(_p(x), _p(out), M, N, _stream(x.device))
    _lib.check(rc, "c3cu_sum_rows_f32_exact")
    return out


def _mm_shapes(A, B, trans_a, trans_b):
    M, K = (A.shape[1], A.shape[0]) if trans_a else (A.shape[0], A.shape[1])
    N = B.shape[0] if trans_b else B.shape[1]
    _f32(B, "B", 2, (N, K) if trans_b else (K, N))
    return M, K, N


def matmul_relu_bwd(A: torch.Tensor, B: torch.Tensor, z: torch.Tensor, trans_a: bool = False,
                    trans_b: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """out = (z > 0 ? 1 : 0) * (A B): the MatMul backward dA followed by the upstream ReLU's
    backward Mul(Gt(z, 0), .), in one launch, bit-exact."""
    _f32(A, "A")
    M, K, N = _mm_shapes(A, B, trans_a, trans_b)
    _f32(z, "z", 2, (M, N))
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    _f32(out, "out", 2, (M, N))
    rc = _lib.load().c3cu_matmul_relu_bwd_f32(_p(A), _p(B), _p(z), _p(out), M, K, N, int(trans_a), int(trans_b),
                                              _stream(A.device))
    _lib.check(rc, "c3cu_matmul_relu_bwd_f32")
    return out


def matmul_colsum(A: torch.Tensor, B: torch.Tensor, trans_a: bool = False, trans_b: bool = False,
                  out: torch.Tensor | None = None, colsum: torch.Tensor | None = None):
    """(A B, column sums of b(k, j) over k): the MatMul backward dB and the Add backward's
    SumReduce of the same gradient, in one launch, bit-exact."""
    _f32(A, "A")
    M, K, N = _mm_shapes(A, B, trans_a, trans_b)
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    if colsum is None:
        colsum = torch.empty(N, dtype=torch.float32, device=A.device)
    _f32(out, "out", 2, (M, N))
    _f32(colsum, "colsum", 1, (N,))
    rc = _lib.load().c3cu_matmul_colsum_f32(_p(A), _p(B), _p(out), _p(colsum), M, K, N, int(trans_a),
                                            int(trans_b), _stream(A.device))
    _lib.check(rc, "c3cu_matmul_colsum_f32")
    return out, colsum
