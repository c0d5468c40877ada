"""Fused Linear+bias+ReLU forward and its captured backward on B200 kernels.

Functional wrappers over the C ABI (include/c3cu.h). Tensors are torch CUDA tensors used
as device memory; every call is launched on torch's current stream of the tensor's
device. Shapes follow the reference region MatMul+Add+ReLU
(include/C3/C3HotPathManager.h:521-611): X [M, K], weight W [N, K] ("nk", nn.Linear) or
B [K, N] ("kn", the reference's MatMul rhs), bias b [N]."""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_ws_cache: dict[tuple[int, int], torch.Tensor] = {}


def _p(t: torch.Tensor | None):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _layout(w_layout: str) -> int:
    if w_layout == "nk":
        return _lib.W_NK
    if w_layout == "kn":
        return _lib.W_KN
    raise ValueError(f"w_layout must be 'nk' or 'kn', got {w_layout!r}")


def _device_ok(t: torch.Tensor) -> bool:
    """Whether an operand lives on a CUDA device (the last check before a C call)."""
    return t.is_cuda


def _require(t: torch.Tensor, name: str, dtype: torch.dtype, ndim: int,
             shape: tuple | None = None):
    """Checks an operand before any C call: dtype, rank, contiguity and (where given) the exact
    shape first, then that it lives on a CUDA device. The C ABI takes bare pointers, so a size
    that disagrees with the allocation would make a kernel or a TMA descriptor reach past it."""
    if not isinstance(t, torch.Tensor):
        raise _lib.C3CUError(-1, name, f"expected a torch.Tensor, got {type(t).__name__}")
    if t.dtype != dtype or t.dim() != ndim or not t.is_contiguous():
        raise _lib.C3CUError(-1, name, f"expected contiguous {dtype} with {ndim} dims, got "
                                       f"{t.dtype} {tuple(t.shape)} contiguous={t.is_contiguous()}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise _lib.C3CUError(-1, name, f"expected shape {tuple(shape)}, got {tuple(t.shape)}")
    if not _device_ok(t):
        raise _lib.C3CUError(-1, name, "expected a CUDA tensor")


def _require_rows(t: torch.Tensor, name: str, dtype: torch.dtype, rows: int, cols: int,
                  min_ld: int | None = None):
    """A row-major 2-D operand that may be a column slice of a wider matrix: shape (rows, cols),
    unit column stride, row stride at least `min_ld` (default cols)."""
    if not isinstance(t, torch.Tensor):
        raise _lib.C3CUError(-1, name, f"expected a torch.Tensor, got {type(t).__name__}")
    if t.dtype != dtype or t.dim() != 2:
        raise _lib.C3CUError(-1, name, f"expected 2-D {dtype}, got {t.dtype} {tuple(t.shape)}")
    if tuple(t.shape) != (rows, cols):
        raise _lib.C3CUError(-1, name, f"expected shape {(rows, cols)}, got {tuple(t.shape)}")
    if rows > 0 and cols > 0 and (t.stride(1) != 1 or (rows > 1 and t.stride(0) < (min_ld or cols))):
        raise _lib.C3CUError(-1, name, f"expected unit column stride and row stride >= {min_ld or cols}, "
                                       f"got strides {t.stride()}")
    if not _device_ok(t):
        raise _lib.C3CUError(-1, name, "expected a CUDA tensor")


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Scratch of the column-sum kernels (per-block partial sums), one buffer per (device,
    stream): launches on different streams never share partials. It is allocated while its
    stream is current, so the caching allocator orders its reuse on that stream."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    ws = _ws_cache.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
        _ws_cache[key] = ws
    return ws


def mask_words(n: int) -> int:
    return (n + 31) // 32


@_lib.on_tensor_device
def forward(X: torch.Tensor, W: torch.Tensor, b: torch.Tensor, w_layout: str = "nk",
            Y: torch.Tensor | None = None, mask: torch.Tensor | None = None):
    """Y = max(X W^T + b, 0) (or X B + b), bf16 out, plus the bit-packed ReLU mask
    ([M, ceil(N/32)] int32 holding uint32 words)."""
    lay = _layout(w_layout)
    _require(X, "X", torch.bfloat16, 2)
    M, K = X.shape
    _require(W, "W", torch.bfloat16, 2)
    N = W.shape[0] if lay == _lib.W_NK else W.shape[1]
    _require(W, "W", torch.bfloat16, 2, (N, K) if lay == _lib.W_NK else (K, N))
    _require(b, "b", torch.float32, 1, (N,))
    if Y is None:
        Y = torch.empty((M, N), dtype=torch.bfloat16, device=X.device)
    _require(Y, "Y", torch.bfloat16, 2, (M, N))
    if mask is None:
        mask = torch.empty((M, mask_words(N)), dtype=torch.int32, device=X.device)
    _require(mask, "mask", torch.int32, 2, (M, mask_words(N)))
    rc = _lib.load().c3cu_linear_bias_relu_fwd(_p(X), _p(W), _p(b), _p(Y), _p(mask), M, N, K, lay,
                                               _stream(X.device))
    _lib.check(rc, "c3cu_linear_bias_relu_fwd")
    return Y, mask


@_lib.on_tensor_device
def relu_mask_db(dY: torch.Tensor, mask: torch.Tensor, dZ: torch.Tensor | None = None,
                 db: torch.Tensor | None = None):
    """dZ = float(mask) * dY (bf16, exact) and db = column sums of dZ (fp32)."""
    _require(dY, "dY", torch.bfloat16, 2)
    M, N = dY.shape
    _require(mask, "mask", torch.int32, 2, (M, mask_words(N)))
    if dZ is None:
        dZ = torch.empty_like(dY)
    _require(dZ, "dZ", torch.bfloat16, 2, (M, N))
    if db is None:
        db = torch.empty(N, dtype=torch.float32, device=dY.device)
    _require(db, "db", torch.float32, 1, (N,))
    L = _lib.load()
    nb = L.c3cu_relu_mask_db_workspace(M, N)
    ws = workspace(dY.device, nb)
    rc = L.c3cu_relu_mask_db(_p(dY), _p(mask), _p(dZ), _p(db), M, N, _p(ws), ws.numel(),
                             _stream(dY.device))
    _lib.check(rc, "c3cu_relu_mask_db")
    return dZ, db


@_lib.on_tensor_device
def grad_input(dZ: torch.Tensor, W: torch.Tensor, w_layout: str = "nk", dX: torch.Tensor | None = None):
    lay = _layout(w_layout)
    _require(dZ, "dZ", torch.bfloat16, 2)
    M, N = dZ.shape
    _require(W, "W", torch.bfloat16, 2)
    K = W.shape[1] if lay == _lib.W_NK else W.shape[0]
    _require(W, "W", torch.bfloat16, 2, (N, K) if lay == _lib.W_NK else (K, N))
    if dX is None:
        dX = torch.empty((M, K), dtype=torch.bfloat16, device=dZ.device)
    _require(dX, "dX", torch.bfloat16, 2, (M, K))
    rc = _lib.load().c3cu_gemm_dx(_p(dZ), _p(W), _p(dX), M, N, K, lay, _stream(dZ.device))
    _lib.check(rc, "c3cu_gemm_dx")
    return dX


@_lib.on_tensor_device
def grad_weight(dZ: torch.Tensor, X: torch.Tensor, w_layout: str = "nk", dW: torch.Tensor | None = None,
                out_dtype: torch.dtype = torch.float32):
    """dW = dZ^T X ([N, K], "nk") or X^T dZ ([K, N], "kn"), fp32 or bf16 (fp32 accumulation)."""
    lay = _layout(w_layout)
    _require(dZ, "dZ", torch.bfloat16, 2)
    M, N = dZ.shape
    _require(X, "X", torch.bfloat16, 2)
    K = X.shape[1]
    _require(X, "X", torch.bfloat16, 2, (M, K))
    shape = (N, K) if lay == _lib.W_NK else (K, N)
    if dW is not None:
        out_dtype = dW.dtype
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise _lib.C3CUError(-1, "dW", f"dW must be float32 or bfloat16, got {out_dtype}")
    if dW is None:
        dW = torch.empty(shape, dtype=out_dtype, device=dZ.device)
    _require_rows(dW, "dW", out_dtype, *shape)
    if out_dtype == torch.float32 and not dW.is_contiguous():
        raise _lib.C3CUError(-1, "dW", "an fp32 dW must be contiguous")
    if out_dtype == torch.bfloat16:
        A, B = (dZ, X) if lay == _lib.W_NK else (X, dZ)
        return gemm(A, B, True, True, _lib.EPI_STORE_BF16, dW, M=shape[0], N=shape[1], K=M)
    rc = _lib.load().c3cu_gemm_dw(_p(dZ), _p(X), _p(dW), M, N, K, lay, _stream(dZ.device))
    _lib.check(rc, "c3cu_gemm_dw")
    return dW


@_lib.on_tensor_device
def backward(dY: torch.Tensor, mask: torch.Tensor, X: torch.Tensor, W: torch.Tensor,
             w_layout: str = "nk"):
    """Captured backward of the region: returns (dX bf16, dW fp32, db fp32)."""
    dZ, db = relu_mask_db(dY, mask)
    dW = grad_weight(dZ, X, w_layout)
    dX = grad_input(dZ, W, w_layout)
    return dX, dW, db


@_lib.on_tensor_device
def gemm(A: torch.Tensor, B: torch.Tensor, a_mn: bool, b_mn: bool, epilogue: int,
         out: torch.Tensor, bias: torch.Tensor | None = None, mask: torch.Tensor | None = None,
         M: int | None = None, N: int | None = None, K: int | None = None):
    """General tcgen05 GEMM out[M, N] = epi(sum_k a(m, k) b(n, k)) (c3cu_gemm_bf16).

    A is [M, K] row-major (a_mn False) or [K, M] (a_mn True); B is [N, K] (b_mn False) or [K, N]
    (b_mn True). Each may be a column slice of a wider matrix (unit column stride). M, N and K
    default to the operand shapes; when given they must agree with them."""
    if epilogue not in (_lib.EPI_BIAS_RELU_MASK, _lib.EPI_STORE_BF16, _lib.EPI_STORE_F32,
                        _lib.EPI_BIAS_STORE_F32):
        raise _lib.C3CUError(-1, "gemm", f"unknown epilogue {epilogue}")
    for t, name in ((A, "A"), (B, "B"), (out, "out")):
        if not isinstance(t, torch.Tensor) or t.dim() != 2:
            raise _lib.C3CUError(-1, name, "expected a 2-D tensor")
    M = (A.shape[1] if a_mn else A.shape[0]) if M is None else M
    K = (A.shape[0] if a_mn else A.shape[1]) if K is None else K
    N = (B.shape[1] if b_mn else B.shape[0]) if N is None else N
    _require_rows(A, "A", torch.bfloat16, *((K, M) if a_mn else (M, K)))
    _require_rows(B, "B", torch.bfloat16, *((K, N) if b_mn else (N, K)))
    out_dtype = torch.bfloat16 if epilogue in (_lib.EPI_BIAS_RELU_MASK, _lib.EPI_STORE_BF16) \
        else torch.float32
    _require_rows(out, "out", out_dtype, M, N)
    if epilogue in (_lib.EPI_BIAS_RELU_MASK, _lib.EPI_BIAS_STORE_F32):
        if bias is None:
            raise _lib.C3CUError(-1, "bias", f"epilogue {epilogue} needs a bias")
        _require(bias, "bias", torch.float32, 1, (N,))
    if epilogue == _lib.EPI_BIAS_RELU_MASK:
        if mask is None:
            raise _lib.C3CUError(-1, "mask", "the ReLU-mask epilogue needs a mask")
        _require_rows(mask, "mask", torch.int32, M, mask_words(N))
    lda = A.stride(0)
    ldb = B.stride(0)
    rc = _lib.load().c3cu_gemm_bf16(_p(A), lda, int(a_mn), _p(B), ldb, int(b_mn), _p(out),
                                    out.stride(0), epilogue, _p(bias), _p(mask),
                                    0 if mask is None else mask.stride(0), M, N, K,
                                    _stream(A.device))
    _lib.check(rc, "c3cu_gemm_bf16")
    return out
