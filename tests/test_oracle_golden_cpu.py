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


def test_oracle_softmax_ce_against_float64():
    rng = np.random.default_rng(3)
    z = (rng.standard_normal((64, 10)) * 3).astype(np.float32)
    y = rng.integers(0, 10, 64).astype(np.int32)
    loss, dz = oracle.softmax_ce(z, y)
    zz = z.astype(np.float64)
    p = np.exp(zz - zz.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    assert abs(loss + np.log(p[np.arange(64), y]).mean()) <= 1e-5 * abs(loss)
    assert np.abs(dz - (p - np.eye(10)[y]) / 64).max() <= 1e-7
    y[5] = 11
    loss_bad, dz_bad = oracle.softmax_ce(z, y)
    assert np.isnan(loss_bad) and np.isnan(dz_bad[5]).all() and not np.isnan(dz_bad[4]).any()


def test_oracle_mlp_step_matches_float64_autodiff():
    """The oracle's composed cfg1 step against a float64 reference of the same math."""
    rng = np.random.default_rng(4)
    sizes = (784, 256, 128, 10)
    params = {}
    for i, (k, n) in enumerate(zip(sizes[:-1], sizes[1:]), start=1):
        b = np.sqrt(6.0 / k)
        params[f"W{i}"] = rng.uniform(-b, b, (k, n)).astype(np.float32)
        params[f"b{i}"] = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    x = rng.uniform(0, 1, (16, 784)).astype(np.float32)
    y = rng.integers(0, 10, 16).astype(np.int32)
    loss, logits, grads, new = oracle.mlp_train_step(params, x, y, 0.01)
    P = {k: v.astype(np.float64) for k, v in params.items()}
    X = x.astype(np.float64)
    z1 = X @ P["W1"] + P["b1"]; a1 = np.maximum(z1, 0)
    z2 = a1 @ P["W2"] + P["b2"]; a2 = np.maximum(z2, 0)
    z3 = a2 @ P["W3"] + P["b3"]
    p = np.exp(z3 - z3.max(1, keepdims=True)); p /= p.sum(1, keepdims=True)
    d3 = (p - np.eye(10)[y]) / 16
    ref = {"W3": a2.T @ d3, "b3": d3.sum(0)}
    d2 = (d3 @ P["W3"].T) * (z2 > 0)
    ref.update(W2=a1.T @ d2, b2=d2.sum(0))
    d1 = (d2 @ P["W2"].T) * (z1 > 0)
    ref.update(W1=X.T @ d1, b1=d1.sum(0))
    for k, v in ref.items():
        assert np.abs(grads[k] - v).max() <= 1e-4 * np.abs(v).max() + 1e-7, k
        assert np.abs(new[k] - (P[k] - 0.01 * v)).max() <= 1e-5, k
