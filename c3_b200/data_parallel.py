"""Data-parallel composition of the captured Linear+bias+ReLU training step.

The reference runs one process on one CPU; its captured backward of the MatMul+Add+ReLU region
(src/C3/C3BackwardCapture.cpp:501-528 ReLU backward, :618-644 Add backward, :681-723 MatMul
backward) is what each rank runs here on its own rows:

    dZ  = mask * dY,  db_r = sum_rows(dZ)          (pre-pass, one kernel)
    dW_r = dZᵀ X                                   (tcgen05 GEMM; bf16 or fp32 out)
    dX  = dZ W                                     (tcgen05 GEMM; needs no exchange)

and the one exchange step of the path is the sum of [dW ‖ db] over the ranks. Rows of X / dY /
mask are split contiguously (`shard_rows`); W and b are replicated. The dW GEMM may run in row
bands of dW (`dw_bands`): each band's all-reduce starts on a communication stream as soon as
its GEMM ends, overlapped with the remaining bands and with the dX GEMM.

`GradientSync` owns one rank's dW / db and sums them:
- "nvls" (default on GPUs, "auto"): the library's in-switch all-reduce on NVLink-multicast memory
  (c3_b200.collective), a separate kernel on a communication stream after the dW GEMM,
  overlapped with dX;
- "fused": the dW GEMM itself sums dW and db over the ranks (c3cu_gemm_dw_allreduce): each
  finished tile of dW is reduced in the NVSwitch while the tensor cores work on the next ones, so
  the exchange needs no separate launch or stream (measured slower than "nvls" on 2 and 8 GPUs);
- "nccl": NCCL through the library's C ABI (c3cu_allreduce_grads on a communicator made by
  c3cu_nccl_comm_init), as a C++ host calls it;
- "group": torch.distributed all_reduce on the process group (NCCL for CUDA tensors, gloo for
  host tensors — the host-side path the CPU tests exercise).

The other paths shard with no exchange at all: the fused forward by rows (`shard_rows`), the
elementwise chain by vector-aligned element ranges (`shard_range`) and the FlashAttention
forward by (batch, head) pairs (`shard_heads`). The cfg1 MLP step sums its gradients with one
all-reduce (c3_b200.mlp.reduce_gradients).
"""
from __future__ import annotations

import os
import sys
from dataclasses import dataclass

import torch
import torch.distributed as dist


def shard_rows(m_global: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous rows [lo, hi) of rank `rank`; the first m_global % world ranks get one more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if m_global < 0:
        raise ValueError("negative row count")
    base, extra = divmod(m_global, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_range(n: int, world: int, rank: int, align: int = 4) -> tuple[int, int]:
    """Contiguous elements [lo, hi) of a flat array of n elements (the cfg4 elementwise chain).
    Every boundary but the last is a multiple of `align` elements (4 fp32 = one 16-byte vector),
    so every shard starts on a vector boundary when the whole array does; the work is split in
    whole vectors, the first ranks taking one more where they do not divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n < 0 or align < 1:
        raise ValueError("negative element count or alignment below 1")
    vecs = (n + align - 1) // align
    lo, hi = shard_rows(vecs, world, rank)
    return min(n, lo * align), min(n, hi * align)


def shard_heads(batch: int, heads: int, world: int, rank: int) -> tuple[int, int]:
    """(batch, head) pairs [lo, hi) of rank `rank`, indexed b * heads + h (the FlashAttention
    forward: every pair is independent). A [B, H, S, D] tensor viewed as [1, B * H, S, D] gives
    the shard as the contiguous slice [:, lo:hi]."""
    if batch < 0 or heads < 0:
        raise ValueError("negative batch or head count")
    return shard_rows(batch * heads, world, rank)


def dw_bands(n: int, chunks: int, align: int = 8) -> list[tuple[int, int]]:
    """Row bands of dW [n, K] for the banded dW GEMM + all-reduce schedule.

    Each band holds a multiple of `align` rows (the bf16 in-switch all-reduce moves 8 elements
    per access and the GEMM's output tile is 8-row aligned); when n does not split into
    `chunks` such bands, one band covers all of dW."""
    if chunks <= 1 or n % (chunks * align) != 0:
        return [(0, n)]
    band = n // chunks
    return [(c * band, (c + 1) * band) for c in range(chunks)]


class GradientSync:
    """dW [N, K] (bf16 or fp32) and db [N] (fp32) of one rank, summed over a process group."""

    def __init__(self, n: int, k: int, device: torch.device, grad_dtype: torch.dtype = torch.bfloat16,
                 collective: str = "auto", group=None, num_ctas: int = 16, peer_frac: float = 0.0,
                 peer_ctas: int = 0):
        """`peer_frac` > 0 (bf16 dW, in-switch collective): that fraction of each dW band is summed
        from peer loads by `peer_ctas` of the `num_ctas` CTAs while the switch sums the rest
        (c3cu_nvls_allreduce_split)."""
        if grad_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError(f"dW dtype must be bfloat16 or float32, got {grad_dtype}")
        if collective not in ("auto", "fused", "nvls", "nccl", "group"):
            raise ValueError(f"collective must be 'auto', 'fused', 'nvls', 'nccl' or 'group', got {collective!r}")
        if collective == "fused" and grad_dtype != torch.bfloat16:
            raise ValueError("the fused dW GEMM + all-reduce writes a bf16 dW")
        self.n, self.k = n, k
        self.device = torch.device(device)
        self.grad_dtype = grad_dtype
        if not 0.0 <= peer_frac <= 1.0 or peer_ctas < 0 or (peer_frac > 0 and not 1 <= peer_ctas < num_ctas):
            raise ValueError(f"peer_frac {peer_frac} / peer_ctas {peer_ctas}: need 0 <= peer_frac <= 1 and, "
                             f"when peer_frac > 0, 1 <= peer_ctas < num_ctas ({num_ctas})")
        self.peer_frac, self.peer_ctas = peer_frac, peer_ctas
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.nvls = None
        self.nccl = None
        want_nvls = collective in ("nvls", "fused") or (collective == "auto" and self.device.type == "cuda"
                                                        and self.world > 1)
        self.fused = False
        if want_nvls:
            try:
                from .collective import NvlsAllReduce
                if grad_dtype == torch.bfloat16:
                    fused = collective == "fused" and n > 128 and k % 8 == 0 and n % 4 == 0
                    words = 4 + 16 * ((n + 255) // 256) * ((k + 255) // 256) if fused else 0
                    self.nvls = NvlsAllReduce(n, self.device, group=group, num_ctas=num_ctas,
                                              numel_bf16=n * k, ar_flag_words=words)
                    self.fused = fused
                    self.dW, self.db = self.nvls.bf16.view(n, k), self.nvls.f32
                else:
                    self.nvls = NvlsAllReduce(n * k + n, self.device, group=group, num_ctas=num_ctas)
                    flat = self.nvls.data()
                    self.dW, self.db = flat[: n * k].view(n, k), flat[n * k:]
            except Exception as exc:
                if collective in ("nvls", "fused"):
                    raise
                print(f"warning: NVLS all-reduce unavailable ({exc}); using the process group",
                      file=sys.stderr)
                self.nvls = None
        if collective == "nccl" and self.world > 1:
            from .collective import NcclComm
            self.nccl = NcclComm(self.device, group)
        self.collective = ("fused" if self.fused else "nvls") if self.nvls is not None else \
            ("nccl" if self.nccl else "group")
        if self.nvls is None:
            if grad_dtype == torch.bfloat16:
                self.dW = torch.empty((n, k), dtype=grad_dtype, device=self.device)
                self.db = torch.empty(n, dtype=torch.float32, device=self.device)
            else:
                flat = torch.empty(n * k + n, dtype=torch.float32, device=self.device)
                self.dW, self.db = flat[: n * k].view(n, k), flat[n * k:]
        self._flat_f32 = None if grad_dtype == torch.bfloat16 else flat

    def gemm_dw_reduce_(self, dZ: torch.Tensor, X: torch.Tensor, stream=None):
        """The fused path: dW = sum over ranks of dZ_rᵀ X_r and db summed in place, one launch."""
        self.nvls.gemm_dw_allreduce_(dZ, X, self.n, self.k, stream)

    def reduce_(self, rows: tuple[int, int] | None = None, with_db: bool = True, stream=None):
        """Sum dW rows [lo, hi) (all rows by default) and, with `with_db`, db over the group.

        Enqueued on `stream` (CUDA tensors; default: the current stream). With one rank this is
        a no-op."""
        if self.world == 1:
            return
        lo, hi = rows if rows is not None else (0, self.n)
        if not 0 <= lo <= hi <= self.n:
            raise ValueError(f"dW rows [{lo}, {hi}) outside [0, {self.n})")
        k, n = self.k, self.n
        if self.nvls is not None:
            if self.grad_dtype == torch.bfloat16:
                if self.peer_frac > 0 and hi > lo:
                    self.nvls.allreduce_split_((lo * k, hi * k), (0, n) if with_db else None, self.peer_frac,
                                               self.peer_ctas, stream)
                else:
                    self.nvls.allreduce2_((lo * k, hi * k) if hi > lo else None,
                                          (0, n) if with_db else None, stream)
            elif with_db and hi == n:
                self.nvls.allreduce_(lo * k, n * k + n, stream)
            else:
                if hi > lo:
                    self.nvls.allreduce_(lo * k, hi * k, stream)
                if with_db:
                    self.nvls.allreduce_(n * k, n * k + n, stream)
            return
        if self.nccl is not None:
            if self._flat_f32 is not None and with_db and hi == n:
                self.nccl.allreduce_(self._flat_f32[lo * k:], stream)
                return
            if hi > lo:
                self.nccl.allreduce_(self.dW[lo:hi], stream)
            if with_db:
                self.nccl.allreduce_(self.db, stream)
            return
        ctx = torch.cuda.stream(stream) if (stream is not None and self.device.type == "cuda") else _Null()
        with ctx:
            if self._flat_f32 is not None and with_db and hi == n:
                dist.all_reduce(self._flat_f32[lo * k:], group=self.group)
                return
            if hi > lo:
                dist.all_reduce(self.dW[lo:hi], group=self.group)
            if with_db:
                dist.all_reduce(self.db, group=self.group)

    def close(self):
        """Releases the NCCL communicator (before the process group is destroyed)."""
        if self.nccl is not None:
            self.nccl.close()
            self.nccl = None


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


@dataclass
class StepEvents:
    """CUDA events of one recorded step: (start, end) per phase on the compute stream and
    (start, end) per all-reduce band on the communication stream."""
    phases: dict
    allreduce: list


class LinearReluTrainStep:
    """The data-parallel captured step of Y = relu(X Wᵀ + b) on one rank's rows.

    forward (Y bf16 + bit-packed ReLU mask) → pre-pass (dZ, db) → dW GEMM in bands, each band's
    all-reduce on `comm` → dX GEMM → the compute stream waits for the last all-reduce.
    `reserve_sms` SMs are left to the collective while the dX GEMM overlaps it. With the
    "fused" collective: forward → pre-pass → dW GEMM that sums dW and db over the ranks → dX."""

    PHASES = ("fwd", "prepass", "dw", "dx")

    def __init__(self, m: int, n: int, k: int, device: torch.device, grad_dtype=torch.bfloat16,
                 collective: str = "auto", group=None, chunks: int = 1, num_ctas: int = 16,
                 reserve_sms: int = 0, overlap_dx: bool = False, peer_frac: float = 0.0, peer_ctas: int = 0):
        from . import _lib
        self.m, self.n, self.k = m, n, k
        self.device = torch.device(device)
        self.sync = GradientSync(n, k, self.device, grad_dtype, collective, group, num_ctas, peer_frac, peer_ctas)
        self.world = self.sync.world
        self.bands = [(0, n)] if self.sync.fused else dw_bands(n, chunks)
        self.reserve_sms = reserve_sms if self.world > 1 else 0
        self.epi = _lib.EPI_STORE_BF16 if grad_dtype == torch.bfloat16 else _lib.EPI_STORE_F32
        dev = self.device
        self.Y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        self.mask = torch.empty((m, (n + 31) // 32), dtype=torch.int32, device=dev)
        self.dZ = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        self.dX = torch.empty((m, k), dtype=torch.bfloat16, device=dev)
        self.comm = torch.cuda.Stream(dev)
        # overlap_dx: dX (which needs only dZ and W) runs on its own stream beside dW, so its tiles
        # fill the SMs that dW's last wave leaves idle
        self.overlap_dx = overlap_dx
        self.side = torch.cuda.Stream(dev) if overlap_dx else None
        self._ev_dz = torch.cuda.Event()
        self._ev_dx = torch.cuda.Event()
        self._ev_band = [torch.cuda.Event() for _ in self.bands]
        self._ev_done = torch.cuda.Event()
        self._sms = torch.cuda.get_device_properties(dev).multi_processor_count

    def close(self):
        self.sync.close()

    @property
    def dW(self) -> torch.Tensor:
        return self.sync.dW

    @property
    def db(self) -> torch.Tensor:
        return self.sync.db

    def __call__(self, X, W, b, dY, record: bool = False) -> StepEvents | None:
        from . import _lib, linear
        comp = torch.cuda.current_stream(self.device)
        phases: dict = {}
        ar: list = []

        def mark(name):
            if record:
                e = torch.cuda.Event(enable_timing=True)
                e.record(comp)
                phases.setdefault(name, []).append(e)

        def mark_on(name, stream):
            if record:
                e = torch.cuda.Event(enable_timing=True)
                e.record(stream)
                phases.setdefault(name, []).append(e)

        def events():
            out = {p: (phases[p][0], phases[p][1]) for p in self.PHASES}
            if "dwdx" in phases:
                out["dwdx"] = (phases["dwdx"][0], phases["dwdx"][1])
            return StepEvents(out, ar)

        mark("fwd"); linear.forward(X, W, b, "nk", self.Y, self.mask); mark("fwd")
        mark("prepass"); linear.relu_mask_db(dY, self.mask, self.dZ, self.db); mark("prepass")
        if self.overlap_dx:
            # dW (with its sum over the ranks when fused) on the compute stream, dX beside it;
            # "dwdx" spans both
            self._ev_dz.record(comp)
            self.side.wait_event(self._ev_dz)
            mark("dwdx")
            mark("dw")
            if self.sync.fused:
                self.sync.gemm_dw_reduce_(self.dZ, X, comp)
            else:
                linear.gemm(self.dZ, X, True, True, self.epi, self.dW, M=self.n, N=self.k, K=self.m)
            mark("dw")
            with torch.cuda.stream(self.side):
                mark_on("dx", self.side)
                linear.grad_input(self.dZ, W, "nk", self.dX)
                mark_on("dx", self.side)
            self._ev_dx.record(self.side)
            comp.wait_event(self._ev_dx)
            mark("dwdx")
            if self.world > 1 and not self.sync.fused:
                self.sync.reduce_((0, self.n), with_db=True, stream=comp)
            return events() if record else None
        mark("dw")
        m, k = self.m, self.k
        if self.sync.fused:
            # dW GEMM and the sum of dW and db over the ranks in one launch; dX follows alone
            self.sync.gemm_dw_reduce_(self.dZ, X, comp)
            mark("dw")
            mark("dx"); linear.grad_input(self.dZ, W, "nk", self.dX); mark("dx")
            return events() if record else None
        lib = _lib.load() if self.reserve_sms else None
        for i, (r0, r1) in enumerate(self.bands):
            # from the second band on, an earlier band's all-reduce runs beside this GEMM: leave
            # it its SMs, as for dX
            if lib is not None and i > 0:
                lib.c3cu_set_gemm_max_ctas(self._sms - self.reserve_sms)
            linear.gemm(self.dZ[:, r0:r1], X, True, True, self.epi, self.dW[r0:r1], M=r1 - r0, N=k, K=m)
            if lib is not None and i > 0:
                lib.c3cu_set_gemm_max_ctas(0)
            if self.world > 1:
                self._ev_band[i].record(comp)
                self.comm.wait_event(self._ev_band[i])
                if record:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e0.record(self.comm)
                self.sync.reduce_((r0, r1), with_db=i == len(self.bands) - 1, stream=self.comm)
                if record:
                    e1 = torch.cuda.Event(enable_timing=True)
                    e1.record(self.comm)
                    ar.append((e0, e1))
        mark("dw")
        if self.world > 1:
            self._ev_done.record(self.comm)
        if lib is not None:
            lib.c3cu_set_gemm_max_ctas(self._sms - self.reserve_sms)
        mark("dx"); linear.grad_input(self.dZ, W, "nk", self.dX); mark("dx")
        if lib is not None:
            lib.c3cu_set_gemm_max_ctas(0)
        if self.world > 1:
            comp.wait_event(self._ev_done)
        return events() if record else None


def default_overlap(world: int) -> tuple[int, int]:
    """(CTAs of the in-switch all-reduce, SMs left free for it during the dX GEMM).

    Measured on B200s (cfg3): 20 CTAs on 20 reserved SMs gave the shortest step with 2 ranks
    (2722 TFLOP/s, against 2370 with no reserve and 16 CTAs) and with 8 ranks (5396 against
    4983). Without a reserve, the all-reduce competes with the CTA-pair dX GEMM's CTAs and
    runs about twice as long. What the reserve costs dX follows from its tile count: 20 SMs
    leave 64 of the 74 CTA pairs, and at 2048 and 4096 rows per rank the 128 and 256 output
    tiles of 256 x 256 take 2 and 4 waves on 64 pairs as on 74, so the reserve is free there;
    at 8192 rows (2 ranks) the 512 tiles take 8 waves instead of 7, which the shorter
    all-reduce more than repays. More CTAs (32 on 32 SMs) cost dX a wave at every size and
    measured slower at 8 ranks; a thread-block cluster per CTA pair changed nothing
    (c3cu_set_collective_cluster)."""
    return (20, 20) if world > 1 else (16, 0)


def env_grad_dtype() -> torch.dtype:
    """C3_GRAD_DTYPE=bf16 (default) | fp32."""
    v = os.environ.get("C3_GRAD_DTYPE", "bf16")
    if v not in ("bf16", "fp32"):
        raise ValueError(f"C3_GRAD_DTYPE must be bf16 or fp32, got {v!r}")
    return torch.bfloat16 if v == "bf16" else torch.float32
