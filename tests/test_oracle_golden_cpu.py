"""Pins the oracle (oracle/c3_oracle.c) to the golden vectors of tests/golden/golden.json, which
an independent Python restatement of the reference's fp32 loops produced
(tests/golden/make_golden.py). Bit-exact except where libm's expf enters (<= 2 ulp)."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "golden.json").read_text())


def arr(v, shape=None):
    a = np.array(v, dtype=np.uint32).view(np.float32)
    return a.reshape(shape) if shape else a


def same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def test_region_forward_golden():
    c = GOLD["region_fwd"]
    M, K, N = c["M"], c["K"], c["N"]
    out, z = oracle.region_fwd(arr(c["X"], (M, K)), arr(c["B"], (K, N)), arr(c["b"]))
    assert same_bits(out, arr(c["out"], (M, N))) and same_bits(z, arr(c["z"], (M, N)))
    c = GOLD["region_fwd_scalar_bias"]
    out, _ = oracle.region_fwd(arr(c["X"], (M, K)), arr(c["B"], (K, N)), arr(c["b"]))
    assert same_bits(out, arr(c["out"], (M, N)))


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_matmul_golden(ta, tb):
    c = GOLD[f"matmul_ta{ta}_tb{tb}"]
    M, K, N = c["M"], c["K"], c["N"]
    A = arr(c["A"], (K, M) if ta else (M, K))
    B = arr(c["B"], (N, K) if tb else (K, N))
    assert same_bits(oracle.matmul(A, B, transA=bool(ta), transB=bool(tb)), arr(c["out"], (M, N)))


def test_matmul_bias_relu_golden():
    c = GOLD["matmul_bias_relu"]
    M, K, N = c["M"], c["K"], c["N"]
    out = oracle.matmul(arr(c["A"], (M, K)), arr(c["B"], (K, N)), bias=arr(c["bias"]), act=1)
    assert same_bits(out, arr(c["out"], (M, N)))


def test_relu_backward_and_sum_reduce_golden():
    c = GOLD["relu_bwd"]
    assert same_bits(oracle.relu_bwd(arr(c["grad"]), arr(c["x"])), arr(c["out"]))
    c = GOLD["sum_reduce_axis0"]
    assert same_bits(oracle.sum_reduce(arr(c["in"], (c["M"], c["N"])), 0), arr(c["out"]))


def test_ew_cfg4_golden():
    c = GOLD["ew_cfg4"]
    out = oracle.ew_cfg4(arr(c["A"]), arr(c["B"]), arr(c["C"]))
    ref = arr(c["out"])
    ulp = np.abs(out.view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
    assert ulp.max() <= 2
