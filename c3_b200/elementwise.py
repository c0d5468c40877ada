"""Single-pass elementwise chains (the reference's FusedNode / linalg.generic kernels,
src/C3/MLIRKernelGen.cpp:394-768, src/C3/LinalgFusedGen.cpp:141-378) on B200."""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from . import linear as _linear
from .linear import _p, _require, _stream, workspace


def _f32_flat(t, name: str, numel: int | None = None):
    """A contiguous fp32 operand (any rank) of `numel` elements when given; checked before
    any C call, since the C ABI trusts the element count it is passed."""
    if not isinstance(t, torch.Tensor):
        raise _lib.C3CUError(-1, name, f"expected a torch.Tensor, got {type(t).__name__}")
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise _lib.C3CUError(-1, name, f"expected a contiguous fp32 tensor, got {t.dtype} "
                                       f"contiguous={t.is_contiguous()}")
    if numel is not None and t.numel() != numel:
        raise _lib.C3CUError(-1, name, f"expected {numel} elements, got {t.numel()}")
    if not _linear._device_ok(t):
        raise _lib.C3CUError(-1, name, "expected a CUDA tensor")

# opcodes of the register-machine encoding (include/c3cu.h, C3CU_EW_*)
ADD, SUB, MUL, DIV, DIV_NANZ, NEG, RELU, EXP, LOG, SIGMOID, TANH, TANH_EXP, GT, CONST, MOV = range(1, 16)


@_lib.on_tensor_device
def chain_cfg4(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, out: torch.Tensor | None = None):
    """out = relu((A + B) * C - A) / (1 + exp(-B)), fp32, one pass over HBM."""
    n = A.numel() if isinstance(A, torch.Tensor) else 0
    for t, name in ((A, "A"), (B, "B"), (C, "C")):
        _f32_flat(t, name, n)
    if out is None:
        out = torch.empty_like(A)
    _f32_flat(out, "out", n)
    rc = _lib.load().c3cu_ew_chain_cfg4(_p(A), _p(B), _p(C), _p(out), A.numel(), _stream(A.device))
    _lib.check(rc, "c3cu_ew_chain_cfg4")
    return out


@_lib.on_tensor_device
def program(inputs: list[torch.Tensor], code: list[tuple[int, int, int, int]], constants: list[float],
            out_reg: int, n: int, out: torch.Tensor | None = None):
    """Runs a register-machine chain: registers 0..len(inputs)-1 hold inputs[i][idx % numel]."""
    if n < 0:
        raise _lib.C3CUError(-1, "program", f"negative element count {n}")
    for i, t in enumerate(inputs):
        _f32_flat(t, f"inputs[{i}]")
        if t.numel() < 1:
            raise _lib.C3CUError(-1, f"inputs[{i}]", "an input needs at least one element "
                                                    "(inputs broadcast as inputs[i][idx % numel])")
    dev = inputs[0].device if inputs else torch.device("cuda")
    if out is None:
        out = torch.empty(n, dtype=torch.float32, device=dev)
    _f32_flat(out, "out")
    if out.numel() < n:
        raise _lib.C3CUError(-1, "out", f"holds {out.numel()} elements, the chain writes {n}")
    ptrs = (ctypes.c_void_p * max(1, len(inputs)))(*[t.data_ptr() for t in inputs])
    nums = (ctypes.c_int64 * max(1, len(inputs)))(*[t.numel() for t in inputs])
    flat = bytes(b for ins in code for b in ins)
    cbuf = (ctypes.c_uint8 * max(1, len(flat)))(*flat)
    consts = (ctypes.c_float * max(1, len(constants)))(*constants)
    rc = _lib.load().c3cu_ew_program(ctypes.cast(ptrs, ctypes.c_void_p), ctypes.cast(nums, ctypes.c_void_p),
                                     len(inputs), ctypes.cast(cbuf, ctypes.c_void_p), len(code),
                                     ctypes.cast(consts, ctypes.c_void_p), len(constants), out_reg,
                                     _p(out), n, _stream(dev))
    _lib.check(rc, "c3cu_ew_program")
    return out


@_lib.on_tensor_device
def sum_rows(x: torch.Tensor, out: torch.Tensor | None = None):
    """Column sums of an fp32 matrix (SumReduce axis 0), deterministic order."""
    _require(x, "x", torch.float32, 2)
    M, N = x.shape
    if out is None:
        out = torch.empty(N, dtype=torch.float32, device=x.device)
    _require(out, "out", torch.float32, 1, (N,))
    L = _lib.load()
    nb = L.c3cu_sum_rows_f32_workspace(M, N)
    ws = workspace(x.device, nb)
    rc = L.c3cu_sum_rows_f32(_p(x), _p(out), M, N, _p(ws), ws.numel(), _stream(x.device))
    _lib.check(rc, "c3cu_sum_rows_f32")
    return out


BW_OPS = {"ReLU": 1, "Sigmoid": 2, "Tanh": 3, "Neg": 4, "Exp": 5, "Log": 6}


@_lib.on_tensor_device
def backward_chain(types: list[str], grad: torch.Tensor, xs: list[torch.Tensor | None],
                   outs: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
    """Fused backward of a chain of unary elementwise nodes (types[0] most downstream):
    returns the gradient each node passes upstream, from one pass (c3cu_ew_backward_chain)."""
    if not types or any(t not in BW_OPS for t in types):
        raise _lib.C3CUError(-1, "backward_chain", f"node types must be a non-empty list of {sorted(BW_OPS)}")
    _f32_flat(grad, "grad")
    n = grad.numel()
    if len(xs) != len(types):
        raise _lib.C3CUError(-1, "xs", f"expected {len(types)} saved inputs (None where unused), got {len(xs)}")
    for i, x in enumerate(xs):
        if x is not None:
            _f32_flat(x, f"xs[{i}]", n)
    if outs is None:
        outs = [torch.empty_like(grad) for _ in types]
    if len(outs) != len(types):
        raise _lib.C3CUError(-1, "outs", f"expected {len(types)} outputs, got {len(outs)}")
    for i, o in enumerate(outs):
        _f32_flat(o, f"outs[{i}]", n)
    ops = (ctypes.c_int * len(types))(*[BW_OPS[t] for t in types])
    xp = (ctypes.c_void_p * len(types))(*[0 if x is None else x.data_ptr() for x in xs])
    op = (ctypes.c_void_p * len(types))(*[o.data_ptr() for o in outs])
    rc = _lib.load().c3cu_ew_backward_chain(ctypes.cast(ops, ctypes.c_void_p), len(types), _p(grad),
                                            ctypes.cast(xp, ctypes.c_void_p), ctypes.cast(op, ctypes.c_void_p),
                                            n, _stream(grad.device))
    _lib.check(rc, "c3cu_ew_backward_chain")
    return outs
