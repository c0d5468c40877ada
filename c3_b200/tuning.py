"""Per-shape kernel selection: the B200 counterpart of the reference's auto-tuner.

The reference searches one global MatMul tile configuration (tile_m / tile_n / tile_k /
unroll) with a QEA optimiser on a 256^3 sample (include/C3/AutoTuner.h:42-63,
src/C3/C3Engine.cpp:1577-1651) and caches compiled kernels on disk under
sha256("c3_jit_<version>_<opt>_<graph>") (src/C3/JITCache.cpp:214-220). Here the kernels are
precompiled; what varies per shape is which GEMM variant runs:
  0  CTA-pair kernel with the split-K tail (automatic)
  1  single-CTA 128 x 256 kernel
  2  CTA-pair kernel without the split
`tune_gemm` times each candidate on the device with CUDA events (after warm-up), keeps the
fastest in the library's per-shape table (c3cu_gemm_tune_set) and in a JSON file keyed like
the reference's JIT cache (sha256 of a versioned description), which `load` re-applies in a
later process.
"""
from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

from . import _lib

VERSION = "c3_tune_v1"
GEMM_VARIANTS = (0, 1, 2)


def default_path() -> Path:
    return Path(os.environ.get("C3_TUNING_CACHE", Path.home() / ".cache" / "c3_b200" / "tuning.json"))


def gemm_key(M: int, N: int, K: int, a_mn: int, b_mn: int, epilogue: int, arch: str = "sm100") -> str:
    desc = f"{VERSION}_{arch}_gemm_{M}x{N}x{K}_a{int(a_mn)}b{int(b_mn)}_e{epilogue}"
    return hashlib.sha256(desc.encode()).hexdigest()


def read(path: str | os.PathLike | None = None) -> dict:
    p = Path(path) if path else default_path()
    if not p.exists():
        return {}
    try:
        data = json.loads(p.read_text())
    except ValueError:
        return {}
    return data if isinstance(data, dict) and data.get("version") == VERSION else {}


def write(entries: dict, path: str | os.PathLike | None = None) -> Path:
    p = Path(path) if path else default_path()
    p.parent.mkdir(parents=True, exist_ok=True)
    data = read(p) or {"version": VERSION, "entries": {}}
    data["entries"].update(entries)
    tmp = p.with_suffix(".tmp")
    tmp.write_text(json.dumps(data, indent=1, sort_keys=True))
    tmp.replace(p)
    return p


def apply(entries: dict) -> int:
    """Installs cached choices in the library's per-shape table; returns how many."""
    L = _lib.load()
    n = 0
    for e in entries.values():
        _lib.check(L.c3cu_gemm_tune_set(e["M"], e["N"], e["K"], e["a_mn"], e["b_mn"], e["epilogue"], e["variant"]),
                   "c3cu_gemm_tune_set")
        n += 1
    return n


def load(path: str | os.PathLike | None = None) -> int:
    return apply(read(path).get("entries", {}))


def tune_gemm(shapes, iters: int = 10, warmup: int = 3, path: str | os.PathLike | None = None,
              persist: bool = True) -> dict:
    """shapes: iterable of (M, N, K, a_mn, b_mn, epilogue) of c3cu_gemm_bf16 calls. Returns
    the entries chosen ({key: {M, N, K, a_mn, b_mn, epilogue, variant, us: {variant: time}}})."""
    import torch
    from . import linear
    L = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    out = {}
    for (M, N, K, a_mn, b_mn, epi) in shapes:
        g = torch.Generator(device=dev).manual_seed(M * 31 + N * 7 + K)
        A = torch.randn((K, M) if a_mn else (M, K), generator=g, device=dev).to(torch.bfloat16)
        B = torch.randn((K, N) if b_mn else (N, K), generator=g, device=dev).to(torch.bfloat16)
        odt = torch.float32 if epi in (2, 3) else torch.bfloat16
        C = torch.empty((M, N), dtype=odt, device=dev)
        bias = torch.zeros(N, device=dev) if epi in (0, 3) else None
        mask = torch.empty((M, (N + 31) // 32), dtype=torch.int32, device=dev) if epi == 0 else None
        times = {}
        for v in GEMM_VARIANTS:
            _lib.check(L.c3cu_gemm_tune_set(M, N, K, a_mn, b_mn, epi, v), "c3cu_gemm_tune_set")
            run = lambda: linear.gemm(A, B, bool(a_mn), bool(b_mn), epi, C, bias=bias, mask=mask, M=M, N=N, K=K)
            for _ in range(warmup):
                run()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            s.record()
            for _ in range(iters):
                run()
            e.record()
            e.synchronize()
            times[v] = s.elapsed_time(e) * 1000.0 / iters
        best = min(times, key=times.get)
        _lib.check(L.c3cu_gemm_tune_set(M, N, K, a_mn, b_mn, epi, best), "c3cu_gemm_tune_set")
        out[gemm_key(M, N, K, a_mn, b_mn, epi)] = {"M": M, "N": N, "K": K, "a_mn": int(a_mn), "b_mn": int(b_mn),
                                                   "epilogue": epi, "variant": best,
                                                   "us": {str(k): round(t, 3) for k, t in times.items()}}
    if persist:
        write(out, path)
    return out
