"""Shared helpers of the parity tests: seeded inputs, bf16 rounding, tolerances."""
from __future__ import annotations

import numpy as np
import torch

# Tolerances: bf16 tensor-core paths <= 2e-2 relative error against an
# fp32 reference; fp32 paths <= 1e-5 relative; ReLU masks bit-exact.
TOL_BF16 = 2e-2
TOL_F32 = 1e-5


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def randn(shape, std, seed, dtype=torch.bfloat16):
    return (torch.randn(shape, generator=gen(seed)) * std).to(dtype)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """Normwise relative error max|out - ref| / max|ref|."""
    scale = float(np.abs(ref).max()) if ref.size else 0.0
    err = float(np.abs(out.astype(np.float64) - ref.astype(np.float64)).max()) if ref.size else 0.0
    return err / scale if scale > 0 else err


def assert_bf16_close(out: np.ndarray, ref: np.ndarray, what: str, tol: float = TOL_BF16):
    """Normwise <= tol, and elementwise |d| <= tol*|ref| + tol*rms(ref)."""
    assert out.shape == ref.shape, (what, out.shape, ref.shape)
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    r = rel_err(out, ref)
    assert r <= tol, f"{what}: normwise relative error {r:.3e} > {tol}"
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2))) if ref.size else 0.0
    bad = np.abs(out - ref) > tol * np.abs(ref) + tol * rms
    assert not bad.any(), f"{what}: {int(bad.sum())} elements outside tol*|ref| + tol*rms"
    return r


def unpack_mask(words: np.ndarray, n: int) -> np.ndarray:
    w = words.astype(np.uint32)
    bits = (w[:, :, None] >> np.arange(32, dtype=np.uint32)) & 1
    return bits.reshape(w.shape[0], -1)[:, :n].astype(bool)


def pack_mask(bits: np.ndarray) -> np.ndarray:
    M, N = bits.shape
    W = (N + 31) // 32
    padded = np.zeros((M, W * 32), dtype=np.uint32)
    padded[:, :N] = bits
    return (padded.reshape(M, W, 32) << np.arange(32, dtype=np.uint32)).sum(axis=2).astype(np.uint32)
