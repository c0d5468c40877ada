"""CPU oracle — TEST INFRASTRUCTURE ONLY.

A restatement of the reference's (ShengFlow/C3) CPU JIT arithmetic for the fused hot path,
used by tests/, __graft_entry__.smoke() and bench.py's CPU baseline as the checker. The
product (c3_b200) never imports it. See c3_oracle.c for the reference file:line each
function follows and for the parity status ("parity unpinned" against reference outputs;
pinned to hand-derived known answers and a second Python restatement under tests/golden/).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_DIR = Path(__file__).resolve().parent
_LIB_PATH = _DIR / "liboracle.so"
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)


def build() -> Path:
    src = _DIR / "c3_oracle.c"
    if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_DIR)], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        sz, i = ctypes.c_size_t, ctypes.c_int
        L.c3o_matmul.argtypes = [_f32p, _f32p, _f32p, sz, sz, sz, i, i, _f32p, sz, i, sz, sz, i]
        L.c3o_region_fwd.argtypes = [_f32p, _f32p, _f32p, sz, _f32p, _f32p, sz, sz, sz, i, sz, sz, i]
        L.c3o_relu_bwd.argtypes = [_f32p, _f32p, _f32p, sz]
        L.c3o_relu_bwd_mask.argtypes = [_f32p, _u32p, sz, _f32p, sz, sz]
        L.c3o_sum_reduce.argtypes = [_f32p, _f32p, sz, sz, i]
        L.c3o_ew_cfg4.argtypes = [_f32p, _f32p, _f32p, _f32p, sz, i]
        L.c3o_ew_program.argtypes = [ctypes.POINTER(_f32p), ctypes.POINTER(ctypes.c_int64), i,
                                     ctypes.POINTER(ctypes.c_uint8), i, _f32p, i, _f32p,
                                     ctypes.c_int64]
        L.c3o_attention_rows.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, sz, sz, ctypes.c_float,
                                         i, sz, sz, _f32p]
        _lib = L
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _null():
    return ctypes.cast(None, _f32p)


def default_threads() -> int:
    return len(os.sched_getaffinity(0))


def matmul(A, B, transA=False, transB=False, bias=None, act=0, rows=None, threads=1, M=None):
    """c3.matmul: out[i,j] = act(bias_j + sum_k a(i,k) b(k,j)), sequential k, no FMA."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    if transA:
        K, Mx = A.shape
    else:
        Mx, K = A.shape
    N = B.shape[0] if transB else B.shape[1]
    M = Mx
    r0, r1 = (0, M) if rows is None else rows
    out = np.zeros((M, N), dtype=np.float32)
    bptr, bn = _null(), 0
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32)
        bptr, bn = _f(bias), bias.size
    lib().c3o_matmul(_f(A), _f(B), _f(out), M, K, N, 112 if transA else 0, 112 if transB else 0,
                     bptr, bn, act, r0, r1, threads)
    return out if rows is None else out[r0:r1]


def region_fwd(X, B, b, transB=False, rows=None, threads=1):
    """MatMul+Add+ReLU region: returns (out, z) for rows [r0, r1) (all rows by default)."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    M, K = X.shape
    N = B.shape[0] if transB else B.shape[1]
    r0, r1 = (0, M) if rows is None else rows
    out = np.zeros((M, N), dtype=np.float32)
    z = np.zeros((M, N), dtype=np.float32)
    lib().c3o_region_fwd(_f(X), _f(B), _f(b), b.size, _f(out), _f(z), M, K, N,
                         112 if transB else 0, r0, r1, threads)
    return out[r0:r1], z[r0:r1]


def relu_bwd(grad, x):
    grad = np.ascontiguousarray(grad, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(grad)
    lib().c3o_relu_bwd(_f(grad), _f(x), _f(out), grad.size)
    return out


def relu_bwd_mask(grad, mask):
    grad = np.ascontiguousarray(grad, dtype=np.float32)
    mask = np.ascontiguousarray(mask, dtype=np.uint32)
    M, N = grad.shape
    out = np.empty_like(grad)
    lib().c3o_relu_bwd_mask(_f(grad), mask.ctypes.data_as(_u32p), mask.shape[1], _f(out), M, N)
    return out


def sum_reduce(x, axis=0):
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, N = x.shape
    out = np.empty(N if axis == 0 else M, dtype=np.float32)
    lib().c3o_sum_reduce(_f(x), _f(out), M, N, axis)
    return out


def ew_cfg4(A, B, C, threads=1):
    A, B, C = (np.ascontiguousarray(t, dtype=np.float32) for t in (A, B, C))
    out = np.empty_like(A)
    lib().c3o_ew_cfg4(_f(A), _f(B), _f(C), _f(out), A.size, threads)
    return out


def ew_program(inputs, code, constants, out_reg, n):
    ins = [np.ascontiguousarray(t, dtype=np.float32).ravel() for t in inputs]
    arr = (_f32p * max(1, len(ins)))(*[_f(t) for t in ins])
    nums = (ctypes.c_int64 * max(1, len(ins)))(*[t.size for t in ins])
    code = np.ascontiguousarray(np.asarray(code, dtype=np.uint8).ravel())
    consts = np.ascontiguousarray(np.asarray(constants if len(constants) else [0.0], dtype=np.float32))
    out = np.empty(n, dtype=np.float32)
    lib().c3o_ew_program(arr, nums, len(ins), code.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                         code.size // 4, _f(consts), out_reg, _f(out), n)
    return out


def attention_rows(q, k, v, scale, causal=True, rows=None):
    """fp32/fp64 textbook attention for one (batch, head); q, k, v: [S, D]."""
    q, k, v = (np.ascontiguousarray(t, dtype=np.float32) for t in (q, k, v))
    S, D = q.shape
    r0, r1 = (0, S) if rows is None else rows
    o = np.zeros((S, D), dtype=np.float32)
    lse = np.zeros(S, dtype=np.float32)
    scratch = np.zeros(S, dtype=np.float32)
    lib().c3o_attention_rows(_f(q), _f(k), _f(v), _f(o), _f(lse), S, D, scale, 1 if causal else 0,
                             r0, r1, _f(scratch))
    return o[r0:r1], lse[r0:r1]


def softmax_ce(z, y):
    """Mean softmax cross-entropy and its gradient w.r.t. the logits (textbook; see c3_oracle.c)."""
    z = np.ascontiguousarray(z, dtype=np.float32)
    y = np.ascontiguousarray(y, dtype=np.int32)
    B, C = z.shape
    loss = np.zeros(1, dtype=np.float32)
    dz = np.empty_like(z)
    lib().c3o_softmax_ce(_f(z), y.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), _f(loss), _f(dz), B, C)
    return float(loss[0]), dz


def sgd(p, g, lr):
    p = np.array(p, dtype=np.float32, copy=True)
    g = np.ascontiguousarray(g, dtype=np.float32)
    lib().c3o_sgd(_f(p), _f(g), p.size, ctypes.c_float(lr))
    return p


def mlp_train_step(params, x, y, lr):
    """One cfg1 training step of the MLP 784 -> 256 -> 128 -> 10 (bias + ReLU on the hidden
    layers, softmax cross-entropy, SGD) composed from the restated kernels, in the order the
    reference's captured path evaluates it:
      forward  z1 = x W1 + b1, a1 = relu(z1)   (MatMul+Add+ReLU region, W as [K, N])
               z2 = a1 W2 + b2, a2 = relu(z2)
               z3 = a2 W3 + b3                 (MatMul with the Add as bias epilogue)
      loss, dz3 = softmax_ce(z3, y)
      backward dW3 = a2^T dz3, db3 = sum_rows dz3, da2 = dz3 W3^T, dz2 = (z2 > 0) * da2, ...
      update   p = p - lr * grad for W1, b1, W2, b2, W3, b3
    params: dict of float32 arrays W1 [784, 256], b1 [256], W2 [256, 128], b2 [128],
    W3 [128, 10], b3 [10]. Returns (loss, logits, grads dict, updated params dict)."""
    W1, b1, W2, b2, W3, b3 = (params[k] for k in ("W1", "b1", "W2", "b2", "W3", "b3"))
    a1, z1 = region_fwd(x, W1, b1)
    a2, z2 = region_fwd(a1, W2, b2)
    z3 = matmul(a2, W3, bias=b3)
    loss, dz3 = softmax_ce(z3, y)
    g = {}
    g["W3"] = matmul(a2, dz3, transA=True)
    g["b3"] = sum_reduce(dz3, 0)
    da2 = matmul(dz3, W3, transB=True)
    dz2 = relu_bwd(da2, z2)
    g["W2"] = matmul(a1, dz2, transA=True)
    g["b2"] = sum_reduce(dz2, 0)
    da1 = matmul(dz2, W2, transB=True)
    dz1 = relu_bwd(da1, z1)
    g["W1"] = matmul(x, dz1, transA=True)
    g["b1"] = sum_reduce(dz1, 0)
    new = {k: sgd(params[k], g[k], lr) for k in params}
    return loss, z3, g, new


BW_OPS = {"ReLU": 1, "Sigmoid": 2, "Tanh": 3, "Neg": 4, "Exp": 5, "Log": 6}


def backward_chain(types, grad, xs):
    """Gradients each node of a unary elementwise chain passes upstream (see c3_oracle.c)."""
    grad = np.ascontiguousarray(grad, dtype=np.float32).ravel()
    n = grad.size
    ops = (ctypes.c_int * len(types))(*[BW_OPS[t] for t in types])
    xs = [None if x is None else np.ascontiguousarray(x, dtype=np.float32).ravel() for x in xs]
    xp = (_f32p * len(types))(*[_null() if x is None else _f(x) for x in xs])
    outs = [np.empty(n, dtype=np.float32) for _ in types]
    op = (_f32p * len(types))(*[_f(o) for o in outs])
    lib().c3o_backward_chain(ops, len(types), _f(grad), xp, op, n)
    return outs
