"""Gradient all-reduce of the data-parallel training step over NVLink.

NvlsAllReduce keeps the gradient buffer in torch symmetric memory, which binds every rank's
copy to one NVLink multicast object, and sums it with the library's in-switch all-reduce
kernels (c3cu_nvls_allreduce, c3cu_nvls_allreduce_f32): each rank reduces its slice through
multimem.ld_reduce and broadcasts it with multimem.st. The buffer has a bf16 region (e.g. dW,
summed with fp32 accumulation in the switch) and an fp32 region (e.g. db, or an fp32 dW).
torch provides the allocation and the multicast mapping (plumbing); the reduction is this
library's kernel.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


def split_point(count: int, peer_frac: float) -> int:
    """First bf16 element of the peer part when the last `peer_frac` of `count` elements (a
    multiple of 8) go to peer loads: a multiple of 8, count when the fraction rounds to nothing."""
    if not 0.0 <= peer_frac <= 1.0:
        raise ValueError(f"peer_frac must be in [0, 1], got {peer_frac}")
    vecs = count // 8
    peer_vecs = int(round(vecs * peer_frac))
    return (vecs - peer_vecs) * 8


class NvlsAllReduce:
    def __init__(self, numel: int, device: torch.device, group=None, num_ctas: int = 32,
                 numel_bf16: int = 0, ar_flag_words: int = 0):
        """numel fp32 elements (region `f32`) and numel_bf16 bf16 elements (region `bf16`), and
        `ar_flag_words` uint32 counters for the fused dW GEMM + all-reduce (c3cu_gemm_dw_allreduce)."""
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group or dist.group.WORLD
        self.numel = numel
        self.numel_bf16 = numel_bf16
        self.num_ctas = num_ctas
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.bf16_off = 0
        self.f32_off = _align(numel_bf16 * 2)
        self.flag_off = _align(self.f32_off + numel * 4)
        self.ar_flags_off = self.flag_off + 256
        self.ar_flag_words = ar_flag_words
        nbytes = self.ar_flags_off + _align(ar_flag_words * 4)
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
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
        if int(self.hdl.buffer_size) < offset + nbytes:
            raise RuntimeError("symmetric allocation smaller than the gradient buffer")
        self.mc = mc_base + offset
        # every rank's copy of this buffer through its unicast address, as mapped in this process
        # (the split all-reduce reads its slice of the peer part from each of them)
        self.peer_bases = [int(self.hdl.buffer_ptrs[r]) + offset for r in range(self.world)]
        self._peer_arr = (ctypes.c_void_p * self.world)(*self.peer_bases)
        self.flag_local = self.buf.data_ptr() + self.flag_off
        self.flag_mc = self.mc + self.flag_off
        self.ar_flags_local = self.buf.data_ptr() + self.ar_flags_off
        self.ar_flags_mc = self.mc + self.ar_flags_off
        self.ar_epoch = 0
        self.f32 = self.buf[self.f32_off:self.f32_off + numel * 4].view(torch.float32)
        self.bf16 = self.buf[self.bf16_off:self.bf16_off + numel_bf16 * 2].view(torch.bfloat16)
        self.epoch = 0
        dist.barrier(group=self.group)
        torch.cuda.synchronize(device)

    def data(self) -> torch.Tensor:
        """The fp32 region."""
        return self.f32

    def allreduce_(self, lo: int = 0, hi: int | None = None, stream: torch.cuda.Stream | None = None):
        """Sum fp32 elements [lo, hi) of the fp32 region over all ranks (any alignment)."""
        hi = self.numel if hi is None else hi
        if not 0 <= lo <= hi <= self.numel:
            raise ValueError(f"fp32 range [{lo}, {hi}) must lie in [0, {self.numel})")
        s = stream or torch.cuda.current_stream(self.buf.device)
        rc = _lib.load().c3cu_nvls_allreduce_f32(ctypes.c_void_p(self.mc + self.f32_off),
                                                 ctypes.c_void_p(self.flag_mc),
                                                 ctypes.c_void_p(self.flag_local), lo, hi, self.rank,
                                                 self.world, self.epoch, self.num_ctas,
                                                 ctypes.c_void_p(s.cuda_stream))
        _lib.check(rc, "c3cu_nvls_allreduce_f32")
        self.epoch += 1

    def _ranges(self, bf16_range, f32_range):
        """Element ranges of the two regions, checked against the regions' sizes (the kernels take
        bare offsets, so a range past a region would reach into the rest of the buffer or past it)."""
        blo, bhi = bf16_range or (0, 0)
        flo, fhi = f32_range or (0, 0)
        if not (0 <= blo <= bhi <= self.numel_bf16 and blo % 8 == 0 and bhi % 8 == 0):
            raise ValueError(f"bf16 range [{blo}, {bhi}) must lie in [0, {self.numel_bf16}) with both ends "
                             "multiples of 8")
        if not (0 <= flo <= fhi <= self.numel and flo % 4 == 0 and fhi % 4 == 0):
            raise ValueError(f"fp32 range [{flo}, {fhi}) must lie in [0, {self.numel}) with both ends "
                             "multiples of 4")
        return blo, bhi, flo, fhi

    def allreduce2_(self, bf16_range=None, f32_range=None, stream: torch.cuda.Stream | None = None):
        """One call summing bf16 elements [lo, hi) (lo, hi multiples of 8) and fp32 elements
        [lo, hi) (multiples of 4) of the two regions."""
        blo, bhi, flo, fhi = self._ranges(bf16_range, f32_range)
        s = stream or torch.cuda.current_stream(self.buf.device)
        rc = _lib.load().c3cu_nvls_allreduce(ctypes.c_void_p(self.mc), ctypes.c_void_p(self.flag_mc),
                                             ctypes.c_void_p(self.flag_local), self.bf16_off + 2 * blo,
                                             bhi - blo, self.f32_off + 4 * flo, fhi - flo, self.rank,
                                             self.world, self.epoch, self.num_ctas,
                                             ctypes.c_void_p(s.cuda_stream))
        _lib.check(rc, "c3cu_nvls_allreduce")
        self.epoch += 1

    def allreduce_split_(self, bf16_range=None, f32_range=None, peer_frac: float = 0.0, peer_ctas: int = 0,
                         stream: torch.cuda.Stream | None = None):
        """allreduce2_ with the last `peer_frac` of the bf16 range (rounded to whole 8-element
        vectors) summed from peer loads by `peer_ctas` of the num_ctas CTAs and the rest in the
        switch (c3cu_nvls_allreduce_split). peer_frac 0 is allreduce2_."""
        blo, bhi, flo, fhi = self._ranges(bf16_range, f32_range)
        count = bhi - blo
        peer_from = split_point(count, peer_frac)
        if peer_from == count:
            self.allreduce2_(bf16_range, f32_range, stream)
            return
        s = stream or torch.cuda.current_stream(self.buf.device)
        rc = _lib.load().c3cu_nvls_allreduce_split(
            ctypes.c_void_p(self.mc), self._peer_arr, ctypes.c_void_p(self.flag_mc),
            ctypes.c_void_p(self.flag_local), self.bf16_off + 2 * blo, count, peer_from, self.f32_off + 4 * flo,
            fhi - flo, self.rank, self.world, self.epoch, self.num_ctas, peer_ctas,
            ctypes.c_void_p(s.cuda_stream))
        _lib.check(rc, "c3cu_nvls_allreduce_split")
        self.epoch += 1


    def gemm_dw_allreduce_(self, dZ: torch.Tensor, X: torch.Tensor, n: int, k: int,
                           stream: torch.cuda.Stream | None = None):
        """dW = sum over ranks of dZ_r^T X_r into the bf16 region ([n, k], nn.Linear layout) and
        db = the sum of the fp32 region's first n elements, in one launch of the fused dW GEMM
        (c3cu_gemm_dw_allreduce). dZ [m, n] and X [m, k] are this rank's rows (bf16)."""
        if self.ar_flag_words < 4 + 16 * ((n + 255) // 256) * ((k + 255) // 256):
            raise ValueError("the buffer was made without enough flag words for this dW shape")
        if self.numel_bf16 < n * k or self.numel < n:
            raise ValueError("dW / db do not fit the buffer's regions")
        m = dZ.shape[0]
        if dZ.shape != (m, n) or X.shape != (m, k) or dZ.dtype != torch.bfloat16 or X.dtype != torch.bfloat16 \
                or not dZ.is_contiguous() or not X.is_contiguous():
            raise ValueError(f"expected contiguous bf16 dZ [{m}, {n}] and X [{m}, {k}]")
        s = stream or torch.cuda.current_stream(self.buf.device)
        rc = _lib.load().c3cu_gemm_dw_allreduce(
            ctypes.c_void_p(dZ.data_ptr()), ctypes.c_void_p(X.data_ptr()),
            ctypes.c_void_p(self.buf.data_ptr() + self.bf16_off), ctypes.c_void_p(self.mc + self.bf16_off),
            ctypes.c_void_p(self.mc + self.f32_off), n, ctypes.c_void_p(self.ar_flags_local),
            ctypes.c_void_p(self.ar_flags_mc), self.ar_flag_words, m, n, k, self.rank, self.world,
            self.ar_epoch, ctypes.c_void_p(s.cuda_stream))
        _lib.check(rc, "c3cu_gemm_dw_allreduce")
        self.ar_epoch += 1


class NcclComm:
    """An NCCL communicator made through the library's C ABI (c3cu_nccl_comm_init) and the
    gradient all-reduce on it (c3cu_allreduce_grads) — the same calls a C++ host of the C3
    API makes. Rank 0's unique id travels to the other ranks over the process group."""

    def __init__(self, device: torch.device, group=None):
        self.group = group or dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.device = torch.device(device)
        L = _lib.load()
        uid = torch.zeros(128, dtype=torch.uint8)
        if self.rank == 0:
            raw = ctypes.create_string_buffer(128)
            _lib.check(L.c3cu_nccl_unique_id(raw), "c3cu_nccl_unique_id")
            uid.copy_(torch.frombuffer(bytearray(raw.raw), dtype=torch.uint8))
        backend = dist.get_backend(self.group)
        t = uid.to(self.device) if backend == "nccl" else uid
        dist.broadcast(t, group_src=0, group=self.group)
        raw = bytes(t.cpu().numpy().tobytes())
        comm = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(L.c3cu_nccl_comm_init(ctypes.byref(comm), raw, self.world, self.rank),
                       "c3cu_nccl_comm_init")
        self.comm = comm

    def allreduce_(self, t: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """In-place sum of a contiguous fp32 or bf16 CUDA tensor over the communicator."""
        if not t.is_cuda or not t.is_contiguous() or t.dtype not in (torch.float32, torch.bfloat16):
            raise _lib.C3CUError(-1, "allreduce_grads", "expected a contiguous fp32/bf16 CUDA tensor")
        s = stream or torch.cuda.current_stream(t.device)
        dt = _lib.DTYPE_F32 if t.dtype == torch.float32 else _lib.DTYPE_BF16
        rc = _lib.load().c3cu_allreduce_grads(ctypes.c_void_p(t.data_ptr()), t.numel(), dt, self.comm,
                                              ctypes.c_void_p(s.cuda_stream))
        _lib.check(rc, "c3cu_allreduce_grads")
        return t

    def close(self):
        if self.comm:
            _lib.check(_lib.load().c3cu_nccl_comm_destroy(self.comm), "c3cu_nccl_comm_destroy")
            self.comm = None
