"""Single-pass elementwise chains (the reference's FusedNode / linalg.generic kernels,
src/C3/MLIRKernelGen.cpp:394-768, src/C3/LinalgFusedGen.cpp:141-378) on B200."""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .linear import _p, _stream, workspace

# opcodes of the register-machine encoding (include/c3cu.h, C3CU_EW_*)
ADD, SUB, MUL, DIV, DIV_NANZ, NEG, RELU, EXP, LOG, SIGMOID, TANH, TANH_EXP, GT, CONST, MOV = range(1, 16)


@_lib.on_tensor_device
def chain_cfg4(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, out: torch.Tensor | None = None):
    """out = relu((A + B) * C - A) / (1 + exp(-B)), fp32, one pass over HBM."""
    for t, n in ((A, "A"), (B, "B"), (C, "C")):
        if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise _lib.C3CUError(-1, n, "expected a contiguous fp32 CUDA tensor")
    if not (A.numel() == B.numel() == C.numel()):
        raise _lib.C3CUError(-1, "chain_cfg4", "size mismatch")
    if out is None:
        out = torch.empty_like(A)
    rc = _lib.load().c3cu_ew_chain_cfg4(_p(A), _p(B), _p(C), _p(out), A.numel(), _stream(A.device))
    _lib.check(rc, "c3cu_ew_chain_cfg4")
    return out


@_lib.on_tensor_device
def program(inputs: list[torch.Tensor], code: list[tuple[int, int, int, int]], constants: list[float],
            out_reg: int, n: int, out: torch.Tensor | None = None):
    """Runs a register-machine chain: registers 0..len(inputs)-1 hold inputs[i][idx % numel]."""
    dev = inputs[0].device if inputs else torch.device("cuda")
    ptrs = (ctypes.c_void_p * max(1, len(inputs)))(*[t.data_ptr() for t in inputs])
    nums = (ctypes.c_int64 * max(1, len(inputs)))(*[t.numel() for t in inputs])
    flat = bytes(b for ins in code for b in ins)
    cbuf = (ctypes.c_uint8 * max(1, len(flat)))(*flat)
    consts = (ctypes.c_float * max(1, len(constants)))(*constants)
    if out is None:
        out = torch.empty(n, dtype=torch.float32, device=dev)
    rc = _lib.load().c3cu_ew_program(ctypes.cast(ptrs, ctypes.c_void_p), ctypes.cast(nums, ctypes.c_void_p),
                                     len(inputs), ctypes.cast(cbuf, ctypes.c_void_p), len(code),
                                     ctypes.cast(consts, ctypes.c_void_p), len(constants), out_reg,
                                     _p(out), n, _stream(dev))
    _lib.check(rc, "c3cu_ew_program")
    return out


@_lib.on_tensor_device
def sum_rows(x: torch.Tensor, out: torch.Tensor | None = None):
    """Column sums of an fp32 matrix (SumReduce axis 0), deterministic order."""
    M, N = x.shape
    if out is None:
        out = torch.empty(N, dtype=torch.float32, device=x.device)
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
    n = grad.numel()
    if outs is None:
        outs = [torch.empty_like(grad) for _ in types]
    ops = (ctypes.c_int * len(types))(*[BW_OPS[t] for t in types])
    xp = (ctypes.c_void_p * len(types))(*[0 if x is None else x.data_ptr() for x in xs])
    op = (ctypes.c_void_p * len(types))(*[o.data_ptr() for o in outs])
    rc = _lib.load().c3cu_ew_backward_chain(ctypes.cast(ops, ctypes.c_void_p), len(types), _p(grad),
                                            ctypes.cast(xp, ctypes.c_void_p), ctypes.cast(op, ctypes.c_void_p),
                                            n, _stream(grad.device))
    _lib.check(rc, "c3cu_ew_backward_chain")
    return outs
