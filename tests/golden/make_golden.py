"""Generates tests/golden/golden.json: small known-answer vectors for the oracle.

An independent restatement of the reference's fp32 arithmetic in plain Python loops over
numpy float32 scalars (every operation rounds to fp32; there is no fused multiply-add),
following the same reference loops as oracle/c3_oracle.c:
  c3.matmul           src/C3/C3DialectLowering.cpp:467-610 (sequential k, fmul then fadd,
                      transA/transB index maps at :546-562, bias-init + act epilogue)
  region forward      src/C3/MLIRKernelGen.cpp:610-768 (T, then maxnum(T + b[idx % nb], 0))
  ReLU backward       src/C3/C3BackwardCapture.cpp:501-528 (Gt(x,0) as 1.0/0.0, times grad)
  SumReduce axis 0    src/C3/C3DialectLowering.cpp:382-465 (rows ascending)
  cfg4 chain          relu((A+B)*C-A)/(1+exp(-B)) in graph order
Values are stored as float32 bit patterns. Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

F = np.float32


def bits(a) -> list[int]:
    return [int(x) for x in np.asarray(a, dtype=np.float32).ravel().view(np.uint32)]


def matmul(A, B, M, K, N, ta, tb, bias=None, act=0):
    out = np.zeros((M, N), np.float32)
    for i in range(M):
        for j in range(N):
            acc = F(0.0) if bias is None else F(bias[0 if bias.size == 1 else j])
            for k in range(K):
                a = A[k, i] if ta else A[i, k]
                b = B[j, k] if tb else B[k, j]
                acc = F(acc + F(a * b))
            if act == 1:
                acc = F(max(acc, F(0.0))) if not np.isnan(acc) else F(0.0)
            out[i, j] = acc
    return out


def region(X, B, b):
    M, K = X.shape
    N = B.shape[1]
    T = matmul(X, B, M, K, N, False, False)
    out = np.zeros_like(T)
    z = np.zeros_like(T)
    for i in range(M):
        for j in range(N):
            idx = i * N + j
            s = F(T[i, j] + b[idx % b.size])
            z[i, j] = s
            out[i, j] = s if s > F(0.0) else F(0.0)
    return out, z


def main():
    rng = np.random.default_rng(20261201)
    cases = {}
    M, K, N = 5, 7, 3
    X = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    b = rng.uniform(-0.5, 0.5, N).astype(np.float32)
    out, z = region(X, B, b)
    cases["region_fwd"] = {"M": M, "K": K, "N": N, "X": bits(X), "B": bits(B), "b": bits(b),
                           "out": bits(out), "z": bits(z)}
    b1 = rng.uniform(-0.5, 0.5, 1).astype(np.float32)
    out1, _ = region(X, B, b1)
    cases["region_fwd_scalar_bias"] = {"M": M, "K": K, "N": N, "X": bits(X), "B": bits(B), "b": bits(b1),
                                       "out": bits(out1)}
    for ta in (0, 1):
        for tb in (0, 1):
            A = rng.uniform(-2, 2, (K, M) if ta else (M, K)).astype(np.float32)
            Bm = rng.uniform(-2, 2, (N, K) if tb else (K, N)).astype(np.float32)
            cases[f"matmul_ta{ta}_tb{tb}"] = {"M": M, "K": K, "N": N, "ta": ta, "tb": tb, "A": bits(A),
                                              "B": bits(Bm), "out": bits(matmul(A, Bm, M, K, N, ta, tb))}
    bias = rng.uniform(-1, 1, N).astype(np.float32)
    A = rng.uniform(-2, 2, (M, K)).astype(np.float32)
    Bm = rng.uniform(-2, 2, (K, N)).astype(np.float32)
    cases["matmul_bias_relu"] = {"M": M, "K": K, "N": N, "A": bits(A), "B": bits(Bm), "bias": bits(bias),
                                 "out": bits(matmul(A, Bm, M, K, N, 0, 0, bias, 1))}
    x = rng.uniform(-1, 1, 24).astype(np.float32)
    x[3] = 0.0
    x[7] = -0.0
    x[11] = np.nan
    g = rng.uniform(-1, 1, 24).astype(np.float32)
    relu = np.array([F(F(1.0) if xi > F(0.0) else F(0.0)) * gi for xi, gi in zip(x, g)], np.float32)
    cases["relu_bwd"] = {"x": bits(x), "grad": bits(g), "out": bits(relu)}
    S = rng.uniform(-1, 1, (6, 4)).astype(np.float32)
    sr = np.zeros(4, np.float32)
    for j in range(4):
        acc = F(0.0)
        for i in range(6):
            acc = F(acc + S[i, j])
        sr[j] = acc
    cases["sum_reduce_axis0"] = {"M": 6, "N": 4, "in": bits(S), "out": bits(sr)}
    n = 16
    a = rng.uniform(-4, 4, n).astype(np.float32)
    bb = rng.uniform(-8, 8, n).astype(np.float32)
    c = rng.uniform(-4, 4, n).astype(np.float32)
    o = np.zeros(n, np.float32)
    for i in range(n):
        d = F(F(1.0) + np.exp(F(-bb[i])))
        t = F(F(F(a[i] + bb[i]) * c[i]) - a[i])
        r = t if t > F(0.0) else F(0.0)
        o[i] = F(r / d)
    cases["ew_cfg4"] = {"A": bits(a), "B": bits(bb), "C": bits(c), "out": bits(o),
                        "note": "contains expf: compare within 2 ulp (libm implementations differ)"}
    path = Path(__file__).resolve().parent / "golden.json"
    path.write_text(json.dumps(cases, indent=0))
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
