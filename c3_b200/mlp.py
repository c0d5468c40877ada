"""The cfg1 MLP training step on the GPU: 784 -> 256 -> 128 -> 10 with bias + ReLU on the
hidden layers, softmax cross-entropy and SGD, fp32, on the bit-exact kernels.

The reference trains this MLP on its CPU JIT (README: MNIST MLP, batch 128): the hidden
layers run as the fused MatMul+Add+ReLU region (include/C3/C3HotPathManager.h:521-611,
src/C3/MLIRKernelGen.cpp:610-768), the output layer as c3.matmul with the Add folded into the
accumulator's initial value (src/C3/MLIRKernelGen.cpp:1091-1201), and the captured backward
(src/C3/C3BackwardCapture.cpp:47-132, 501-528, 618-644, 681-723) as transposed c3.matmul,
Mul(Gt(z, 0), grad) and SumReduce. Each of those runs here on the kernel that reproduces the
reference's fp32 loop order bit for bit (c3cu_region_fwd_f32, c3cu_matmul_f32,
c3cu_ew_program, c3cu_sum_rows_f32_exact). The loss and the optimizer belong to the
reference's host framework (not in its sources): c3cu_softmax_ce_f32 and c3cu_sgd_f32 use the
textbook definitions.

Weights use the reference's MatMul layout W [K, N] (fan_in rows). A step is 15 launches on
the current stream; `capture()` records them once in a CUDA graph so that a step costs one
graph launch.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from . import elementwise as ew

LAYERS = (784, 256, 128, 10)
PARAM_NAMES = ("W1", "b1", "W2", "b2", "W3", "b3")

# Mul(Gt(z, 0), grad): registers 0 = z, 1 = grad, 2 = constant 0 (table entry 0); the result
# in register 3
_RELU_BWD = [(ew.CONST, 2, 0, 0), (ew.GT, 3, 0, 2), (ew.MUL, 3, 3, 1)]


def init_params(seed: int = 1234, device: torch.device | str = "cpu", layers=LAYERS) -> dict:
    """Kaiming-uniform weights (bound sqrt(6 / fan_in)) and zero biases, fp32."""
    g = torch.Generator().manual_seed(seed)
    p = {}
    for i, (k, n) in enumerate(zip(layers[:-1], layers[1:]), start=1):
        bound = math.sqrt(6.0 / k)
        p[f"W{i}"] = ((torch.rand((k, n), generator=g) * 2 - 1) * bound).to(device)
        p[f"b{i}"] = torch.zeros(n).to(device)
    return p


def synthetic_batch(seed: int, batch: int = 128, device: torch.device | str = "cpu", classes: int = 10):
    """x ~ U[0, 1] of shape [batch, 784], labels ~ U{0..classes-1} (int32)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.rand((batch, LAYERS[0]), generator=g)
    y = torch.randint(0, classes, (batch,), generator=g, dtype=torch.int32)
    return x.to(device), y.to(device)


class MLPTrainStep:
    """One training step of the cfg1 MLP on device-resident fp32 parameters (updated in
    place). Buffers are allocated once, so a step can be replayed from a CUDA graph."""

    def __init__(self, params: dict, batch: int, lr: float = 0.01):
        self.p = params
        for k in PARAM_NAMES:
            t = params[k]
            if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
                raise _lib.C3CUError(-1, "MLPTrainStep", f"{k}: expected a contiguous fp32 CUDA tensor")
        self.B = batch
        self.lr = float(lr)
        dev = params["W1"].device
        self.device = dev
        d0, d1, d2, d3 = LAYERS
        f = lambda *s: torch.empty(s, dtype=torch.float32, device=dev)
        self.a1, self.z1 = f(batch, d1), f(batch, d1)
        self.a2, self.z2 = f(batch, d2), f(batch, d2)
        self.z3, self.dz3 = f(batch, d3), f(batch, d3)
        self.loss = f(1)
        self.da2, self.dz2 = f(batch, d2), f(batch, d2)
        self.da1, self.dz1 = f(batch, d1), f(batch, d1)
        self.g = {k: torch.empty_like(params[k]) for k in PARAM_NAMES}
        n = len(PARAM_NAMES)
        self._pp = (ctypes.c_void_p * n)(*[params[k].data_ptr() for k in PARAM_NAMES])
        self._gp = (ctypes.c_void_p * n)(*[self.g[k].data_ptr() for k in PARAM_NAMES])
        self._np = (ctypes.c_int64 * n)(*[params[k].numel() for k in PARAM_NAMES])
        self.graph = None

    # ------------------------------------------------------------------ kernels
    def _mm(self, A, B, out, M, K, N, ta, tb, bias=None):
        L = _lib.load()
        rc = L.c3cu_matmul_f32(ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                               ctypes.c_void_p(out.data_ptr()), M, K, N, ta, tb,
                               ctypes.c_void_p(0 if bias is None else bias.data_ptr()),
                               0 if bias is None else bias.numel(), 0, self._stream())
        _lib.check(rc, "c3cu_matmul_f32")

    def _region(self, X, W, b, out, z, M, K, N):
        # the pre-activation z feeds the ReLU backward; no bit mask is needed (and none is built)
        rc = _lib.load().c3cu_region_fwd_f32(ctypes.c_void_p(X.data_ptr()), ctypes.c_void_p(W.data_ptr()),
                                             ctypes.c_void_p(b.data_ptr()), b.numel(),
                                             ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(z.data_ptr()),
                                             ctypes.c_void_p(0), M, K, N, 0, self._stream())
        _lib.check(rc, "c3cu_region_fwd_f32")

    def _colsum(self, x, out, M, N):
        rc = _lib.load().c3cu_sum_rows_f32_exact(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                                 M, N, self._stream())
        _lib.check(rc, "c3cu_sum_rows_f32_exact")

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    # ------------------------------------------------------------------ the step
    def step(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        """Forward, loss, backward and SGD update for one batch; returns the device scalar loss."""
        if x.shape != (self.B, LAYERS[0]) or x.dtype != torch.float32 or not x.is_contiguous():
            raise _lib.C3CUError(-1, "MLPTrainStep.step", f"x must be contiguous fp32 [{self.B}, {LAYERS[0]}]")
        if y.shape != (self.B,) or y.dtype != torch.int32:
            raise _lib.C3CUError(-1, "MLPTrainStep.step", f"y must be int32 [{self.B}]")
        B = self.B
        d0, d1, d2, d3 = LAYERS
        p, g = self.p, self.g
        # forward
        self._region(x, p["W1"], p["b1"], self.a1, self.z1, B, d0, d1)
        self._region(self.a1, p["W2"], p["b2"], self.a2, self.z2, B, d1, d2)
        self._mm(self.a2, p["W3"], self.z3, B, d2, d3, 0, 0, bias=p["b3"])
        rc = _lib.load().c3cu_softmax_ce_f32(ctypes.c_void_p(self.z3.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                             ctypes.c_void_p(self.loss.data_ptr()),
                                             ctypes.c_void_p(self.dz3.data_ptr()), B, d3, self._stream())
        _lib.check(rc, "c3cu_softmax_ce_f32")
        # backward (captured-gradient order: output layer first)
        self._mm(self.a2, self.dz3, g["W3"], d2, B, d3, 1, 0)
        self._colsum(self.dz3, g["b3"], B, d3)
        self._mm(self.dz3, p["W3"], self.da2, B, d3, d2, 0, 1)
        ew.program([self.z2, self.da2], _RELU_BWD, [0.0], 3, B * d2, out=self.dz2)
        self._mm(self.a1, self.dz2, g["W2"], d1, B, d2, 1, 0)
        self._colsum(self.dz2, g["b2"], B, d2)
        self._mm(self.dz2, p["W2"], self.da1, B, d2, d1, 0, 1)
        ew.program([self.z1, self.da1], _RELU_BWD, [0.0], 3, B * d1, out=self.dz1)
        self._mm(x, self.dz1, g["W1"], d0, B, d1, 1, 0)
        self._colsum(self.dz1, g["b1"], B, d1)
        # update
        rc = _lib.load().c3cu_sgd_f32(ctypes.cast(self._pp, ctypes.c_void_p), ctypes.cast(self._gp, ctypes.c_void_p),
                                      ctypes.cast(self._np, ctypes.c_void_p), len(PARAM_NAMES),
                                      ctypes.c_float(self.lr), self._stream())
        _lib.check(rc, "c3cu_sgd_f32")
        return self.loss

    def capture(self):
        """Records one step on static input buffers (`self.x_static`, `self.y_static`) in a CUDA
        graph; `replay()` then runs a step as a single graph launch."""
        self.x_static = torch.zeros((self.B, LAYERS[0]), dtype=torch.float32, device=self.device)
        self.y_static = torch.zeros((self.B,), dtype=torch.int32, device=self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):  # capturing records the launches; nothing runs
            with torch.cuda.graph(self.graph, stream=side):
                self.step(self.x_static, self.y_static)
        torch.cuda.current_stream(self.device).wait_stream(side)
        return self.graph

    def replay(self, x: torch.Tensor | None = None, y: torch.Tensor | None = None) -> torch.Tensor:
        if self.graph is None:
            raise RuntimeError("capture() first")
        if x is not None:
            self.x_static.copy_(x)
        if y is not None:
            self.y_static.copy_(y)
        self.graph.replay()
        return self.loss
