"""Gradient all-reduce of the data-parallel training step over NVLink.

NvlsAllReduce keeps an fp32 buffer (the packed [dW | db] gradients) in torch symmetric
memory, which binds every rank's copy to one NVLink multicast object, and sums it with the
library's in-switch all-reduce kernel (c3cu_nvls_allreduce_f32): each rank reduces its slice
through multimem.ld_reduce and broadcasts it with multimem.st. torch provides the allocation
and the multicast mapping (plumbing); the reduction is this library's kernel.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

_FLAG_PAD = 64  # floats after the data: one uint32 barrier counter on its own 256 B


class NvlsAllReduce:
    def __init__(self, numel: int, device: torch.device, group=None, num_ctas: int = 32):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group or dist.group.WORLD
        self.numel = numel
        self.num_ctas = num_ctas
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.buf = symm_mem.empty(numel + _FLAG_PAD, dtype=torch.float32, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        self.hdl = symm_mem.rendezvous(self.buf, self.group)
        mc_base = int(self.hdl.multicast_ptr)
        if mc_base == 0:
            raise RuntimeError("NVLink multicast is not available for this process group")
        # The handle describes the whole symmetric allocation; this tensor sits `offset`
        # bytes into it (the same offset on every rank and in the multicast mapping).
        offset = int(getattr(self.hdl, "offset", 0))
        local_base = int(self.hdl.buffer_ptrs[self.rank])
        if offset == 0 and local_base != self.buf.data_ptr():
            offset = self.buf.data_ptr() - local_base
        if local_base + offset != self.buf.data_ptr():
            raise RuntimeError("symmetric buffer pointers are inconsistent "
                               f"(base {local_base:#x} + offset {offset} != {self.buf.data_ptr():#x})")
        if int(self.hdl.buffer_size) < offset + (numel + _FLAG_PAD) * 4:
            raise RuntimeError("symmetric allocation smaller than the gradient buffer")
        self.mc = mc_base + offset
        self.flag_local = self.buf.data_ptr() + numel * 4
        self.flag_mc = self.mc + numel * 4
        self.epoch = 0
        dist.barrier(group=self.group)
        torch.cuda.synchronize(device)

    def data(self) -> torch.Tensor:
        return self.buf[: self.numel]

    def allreduce_(self, lo: int = 0, hi: int | None = None, stream: torch.cuda.Stream | None = None):
        hi = self.numel if hi is None else hi
        s = stream or torch.cuda.current_stream(self.buf.device)
        rc = _lib.load().c3cu_nvls_allreduce_f32(ctypes.c_void_p(self.mc), ctypes.c_void_p(self.flag_mc),
                                                 ctypes.c_void_p(self.flag_local), lo, hi, self.rank,
                                                 self.world, self.epoch, self.num_ctas,
                                                 ctypes.c_void_p(s.cuda_stream))
        _lib.check(rc, "c3cu_nvls_allreduce_f32")
        self.epoch += 1
