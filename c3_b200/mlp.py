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

Weights use the reference's MatMul layout W [K, N] (fan_in rows). A step is 10 launches on
the current stream (each MatMul backward fused with its neighbouring ReLU or Add backward);
`capture()` records them once in a CUDA graph so that a step costs one graph launch.

Data parallel (one process per GPU): each rank runs the step on its equal share of the global
batch (`shard_batch`). The gradients and the loss share one flat fp32 buffer, so one all-reduce
(sum) per step covers them; SGD then uses lr / world and the loss slot is scaled by 1 / world,
which gives the full-batch mean gradient and mean loss (each rank's loss is already the mean of
its rows). W and b stay replicated; all ranks apply the same update.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist

from . import _lib
from .data_parallel import shard_rows

LAYERS = (784, 256, 128, 10)
PARAM_NAMES = ("W1", "b1", "W2", "b2", "W3", "b3")


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


def shard_batch(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of the global batch that rank `rank` trains on. The shares must be equal:
    each rank's loss is the mean over its own rows, and the sum over ranks is rescaled by
    1 / world."""
    if world < 1 or global_batch % world != 0:
        raise ValueError(f"a global batch of {global_batch} does not split evenly over {world} ranks")
    return shard_rows(global_batch, world, rank)


_SEGMENT_ALIGN = 64  # elements (256 bytes): every gradient view starts on a 256-byte boundary


def _segments(shapes: dict) -> list[tuple[int, int]]:
    """(offset, numel) of each gradient in PARAM_NAMES order, then of the loss."""
    out, off = [], 0
    for n in [math.prod(shapes[k]) for k in PARAM_NAMES] + [1]:
        out.append((off, n))
        off += (n + _SEGMENT_ALIGN - 1) // _SEGMENT_ALIGN * _SEGMENT_ALIGN
    return out


def flat_numel(shapes: dict) -> int:
    off, n = _segments(shapes)[-1]
    return off + n


def gradient_views(flat: torch.Tensor, shapes: dict) -> tuple[dict, torch.Tensor]:
    """Views of one flat fp32 buffer: the gradient of each parameter in PARAM_NAMES order,
    then the loss (1 element, the buffer's last). Each view starts on a 256-byte boundary;
    `flat` must hold flat_numel(shapes) elements."""
    if flat.numel() != flat_numel(shapes) or not flat.is_contiguous():
        raise ValueError(f"flat buffer holds {flat.numel()} elements, the layout needs {flat_numel(shapes)}")
    seg = _segments(shapes)
    views = {k: flat[o:o + n].view(shapes[k]) for k, (o, n) in zip(PARAM_NAMES, seg)}
    o, n = seg[-1]
    return views, flat[o:o + n]


def reduce_gradients(flat: torch.Tensor, world: int, group=None) -> None:
    """Sums the gradient + loss buffer over the ranks and turns the loss slot into the mean of
    the ranks' losses. The gradients stay summed; the update uses `data_parallel_lr`."""
    if world <= 1:
        return
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    flat[-1:].mul_(1.0 / world)


def data_parallel_lr(lr: float, world: int) -> float:
    """SGD step on the summed gradients of `world` equal shards (each a mean over its rows)."""
    return float(lr) / world


class MLPTrainStep:
    """One training step of the cfg1 MLP on device-resident fp32 parameters (updated in
    place). Buffers are allocated once, so a step can be replayed from a CUDA graph.

    `batch` is this process's batch. With `group` (a torch.distributed process group whose
    size is above 1; dist.group.WORLD for the default one) the step is data parallel: the
    gradients and the loss are summed over the group before the update."""

    def __init__(self, params: dict, batch: int, lr: float = 0.01, group=None):
        self.p = params
        for k in PARAM_NAMES:
            t = params[k]
            if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
                raise _lib.C3CUError(-1, "MLPTrainStep", f"{k}: expected a contiguous fp32 CUDA tensor")
        self.B = batch
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.lr = float(lr)
        self.lr_step = data_parallel_lr(lr, self.world)
        dev = params["W1"].device
        self.device = dev
        d0, d1, d2, d3 = LAYERS
        f = lambda *s: torch.empty(s, dtype=torch.float32, device=dev)
        self.a1, self.z1 = f(batch, d1), f(batch, d1)
        self.a2, self.z2 = f(batch, d2), f(batch, d2)
        self.z3, self.dz3 = f(batch, d3), f(batch, d3)
        self.dz2 = f(batch, d2)
        self.dz1 = f(batch, d1)
        # gradients and loss in one buffer: one all-reduce covers them under data parallelism
        shapes = {k: tuple(params[k].shape) for k in PARAM_NAMES}
        self.flat = torch.zeros(flat_numel(shapes), dtype=torch.float32, device=dev)
        self.g, self.loss = gradient_views(self.flat, shapes)
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

    def _mm_colsum(self, A, G, dW, db, M, K, N):
        # dW [M, N] = A^T G (A stored [K, M]) and db = column sums of G [K, N]
        rc = _lib.load().c3cu_matmul_colsum_f32(ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(G.data_ptr()),
                                                ctypes.c_void_p(dW.data_ptr()), ctypes.c_void_p(db.data_ptr()),
                                                M, K, N, 1, 0, self._stream())
        _lib.check(rc, "c3cu_matmul_colsum_f32")

    def _mm_relu_bwd(self, G, W, z, dz, M, K, N):
        # dz [M, N] = (z > 0) * (G W^T), G [M, K], W [N, K]
        rc = _lib.load().c3cu_matmul_relu_bwd_f32(ctypes.c_void_p(G.data_ptr()), ctypes.c_void_p(W.data_ptr()),
                                                  ctypes.c_void_p(z.data_ptr()), ctypes.c_void_p(dz.data_ptr()),
                                                  M, K, N, 0, 1, self._stream())
        _lib.check(rc, "c3cu_matmul_relu_bwd_f32")

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    # ------------------------------------------------------------------ the step
    def step(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        """Forward, loss, backward and SGD update for one batch; returns the device scalar loss.
        Runs on the parameters' device whichever device is current."""
        with torch.cuda.device(self.device):
            return self._step(x, y)

    def _step(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        if x.device != self.device or y.device != self.device:
            raise _lib.C3CUError(-1, "MLPTrainStep.step", f"x and y must be on {self.device}")
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
        # backward (captured-gradient order: output layer first), each MatMul backward fused
        # with its neighbour: dW with the Add backward's SumReduce (db), dA with the upstream
        # ReLU backward (dz = (z > 0) * dA); 5 launches instead of 10, the same bits
        self._mm_colsum(self.a2, self.dz3, g["W3"], g["b3"], d2, B, d3)
        self._mm_relu_bwd(self.dz3, p["W3"], self.z2, self.dz2, B, d3, d2)
        self._mm_colsum(self.a1, self.dz2, g["W2"], g["b2"], d1, B, d2)
        self._mm_relu_bwd(self.dz2, p["W2"], self.z1, self.dz1, B, d2, d1)
        self._mm_colsum(x, self.dz1, g["W1"], g["b1"], d0, B, d1)
        # the one exchange step under data parallelism (NCCL for CUDA tensors)
        reduce_gradients(self.flat, self.world, self.group)
        # update
        rc = _lib.load().c3cu_sgd_f32(ctypes.cast(self._pp, ctypes.c_void_p), ctypes.cast(self._gp, ctypes.c_void_p),
                                      ctypes.cast(self._np, ctypes.c_void_p), len(PARAM_NAMES),
                                      ctypes.c_float(self.lr_step), self._stream())
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
