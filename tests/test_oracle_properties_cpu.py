"""Property tests of the oracle (oracle/c3_oracle.c, test infrastructure) over random shapes,
against independent numpy restatements of the reference's fp32 loops:

- c3.matmul (src/C3/C3DialectLowering.cpp:467-610): out[i,j] = ((0 + a_i0*b_0j) + a_i1*b_1j) + ...,
  k ascending, a separate fp32 rounding after every multiply and every add. numpy float32
  arithmetic rounds each elementwise operation to fp32, so a k loop over float32 arrays is the
  same computation; transposes only change the indexing (transA: A stored [K, M]; transB: B
  stored [N, K]).
- the region (src/C3/MLIRKernelGen.cpp:610-768): z = T + b[j % numel(b)], out = maxnum(z, 0).
- ReLU backward Mul(Gt(x, 0), grad) (src/C3/C3BackwardCapture.cpp:501-528) and SumReduce axis 0,
  i ascending (src/C3/C3DialectLowering.cpp:382-465).
- the fused backward chains: the reference's per-type gradient graphs chained upstream, with
  libm's expf (called through ctypes, as the reference's JIT calls it).

All comparisons are bit-exact."""
import ctypes
import ctypes.util

import numpy as np
from hypothesis import given, settings, strategies as st

import oracle


def _seq_k_matmul(A, B, ta, tb):
    A = A.T if ta else A  # logical [M, K]
    B = B.T if tb else B  # logical [K, N]
    M, K = A.shape
    N = B.shape[1]
    acc = np.zeros((M, N), np.float32)
    for k in range(K):
        acc = acc + A[:, k:k + 1] * B[k:k + 1, :]  # float32 multiply, then float32 add
    return acc


def _rand(rng, shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float32)


def _bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@settings(max_examples=60, deadline=None)
@given(M=st.integers(1, 24), K=st.integers(1, 40), N=st.integers(1, 24), ta=st.booleans(), tb=st.booleans(),
       seed=st.integers(0, 2 ** 31 - 1))
def test_matmul_is_sequential_k_fp32(M, K, N, ta, tb, seed):
    rng = np.random.default_rng(seed)
    A = _rand(rng, (K, M) if ta else (M, K))
    B = _rand(rng, (N, K) if tb else (K, N))
    out = oracle.matmul(A, B, transA=ta, transB=tb)
    assert _bits_equal(out, _seq_k_matmul(A, B, ta, tb))


@settings(max_examples=60, deadline=None)
@given(M=st.integers(1, 24), K=st.integers(1, 40), N=st.integers(1, 24),
       bias_kind=st.sampled_from(["row", "scalar"]), seed=st.integers(0, 2 ** 31 - 1))
def test_region_is_bias_after_the_k_sum_then_maxnum(M, K, N, bias_kind, seed):
    rng = np.random.default_rng(seed)
    X, B = _rand(rng, (M, K)), _rand(rng, (K, N), 0.3)
    b = _rand(rng, (N,) if bias_kind == "row" else (1,), 0.1)
    out, z = oracle.region_fwd(X, B, b)
    T = _seq_k_matmul(X, B, False, False)
    z_ref = T + np.broadcast_to(b, (N,)) if b.size == N else T + b[0]
    assert _bits_equal(z, z_ref)
    # maxnum(z, 0): z where z > 0, else +0 or -0; compare values (signed zeros both count as 0)
    ref = np.where(z_ref > 0, z_ref, np.float32(0))
    assert np.array_equal(out, ref)


@settings(max_examples=60, deadline=None)
@given(M=st.integers(1, 64), N=st.integers(1, 48), seed=st.integers(0, 2 ** 31 - 1))
def test_relu_backward_and_sum_reduce_orders(M, N, seed):
    rng = np.random.default_rng(seed)
    grad, x = _rand(rng, (M, N)), _rand(rng, (M, N))
    x[rng.random((M, N)) < 0.1] = 0.0  # Gt(0, 0) is false: the gradient is zeroed
    dz = oracle.relu_bwd(grad, x)
    dz_ref = np.where(x > 0, np.float32(1), np.float32(0)) * grad
    assert _bits_equal(dz, dz_ref)
    db = oracle.sum_reduce(np.ascontiguousarray(dz.reshape(M, N)), 0)
    acc = np.zeros(N, np.float32)
    for i in range(M):
        acc = acc + dz_ref.reshape(M, N)[i]
    assert _bits_equal(db, acc)


_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]
_expf_v = np.vectorize(lambda v: _libm.expf(v), otypes=[np.float32])


def _expf(x):
    # libm's expf, the function the reference's JIT calls (math.exp lowers to it)
    return _expf_v(x.astype(np.float32)).astype(np.float32)


def _chain_ref(types, grad, xs):
    """The reference's per-type backward graphs (src/C3/C3BackwardCapture.cpp:501-617 ReLU,
    Sigmoid, Tanh; 725-743 Neg; 823-872 Exp, Log), one fp32 operation per graph node, chained
    from the most downstream node upstream."""
    g = grad.astype(np.float32)
    outs = []
    one = np.float32(1)
    for t, x in zip(types, xs):
        x = np.zeros_like(g) if x is None else x.astype(np.float32)
        if t == "ReLU":
            r = np.where(x > 0, one, np.float32(0)) * g
        elif t == "Sigmoid":
            s = one / (one + _expf(-x))
            r = g * (s * (one - s))
        elif t == "Tanh":
            ep, en = _expf(x), _expf(-x)
            th = (ep - en) / (ep + en)
            r = g * (one - th * th)
        elif t == "Neg":
            r = -g
        elif t == "Exp":
            r = _expf(x) * g
        elif t == "Log":
            r = g / x
        outs.append(r.astype(np.float32))
        g = outs[-1]
    return outs


@settings(max_examples=80, deadline=None)
@given(types=st.lists(st.sampled_from(["ReLU", "Sigmoid", "Tanh", "Neg", "Exp", "Log"]), min_size=1, max_size=5),
       n=st.integers(1, 300), seed=st.integers(0, 2 ** 31 - 1))
def test_backward_chain_follows_the_per_type_graphs(types, n, seed):
    rng = np.random.default_rng(seed)
    grad = _rand(rng, (n,))
    # Log's input away from 0; Exp/Tanh/Sigmoid inputs in a range where exp stays finite
    xs = [(rng.random(n).astype(np.float32) + np.float32(0.5)) if t == "Log" else _rand(rng, (n,), 2.0)
          for t in types]
    got = oracle.backward_chain(types, grad, xs)
    ref = _chain_ref(types, grad, xs)
    for k, (g, r) in enumerate(zip(got, ref)):
        assert _bits_equal(g, r), (types, k, float(np.abs(g - r).max()))


_libm.logf.restype = ctypes.c_float
_libm.logf.argtypes = [ctypes.c_float]


@settings(max_examples=60, deadline=None)
@given(n=st.integers(1, 2000), threads=st.sampled_from([1, 3, 8]), seed=st.integers(0, 2 ** 31 - 1))
def test_cfg4_chain_elementwise_order(n, threads, seed):
    """relu((A + B) * C - A) / (1 + exp(-B)) (MLIRKernelGen.cpp:610-768 scalar fused path):
    Neg, Exp, Add, Add, Mul, Sub, ReLU = maxnum(x, 0), Div, one fp32 operation each; the result
    does not depend on how the elements are split over host threads."""
    rng = np.random.default_rng(seed)
    A = (rng.random(n) * 8 - 4).astype(np.float32)
    B = (rng.random(n) * 16 - 8).astype(np.float32)
    C = (rng.random(n) * 8 - 4).astype(np.float32)
    out = oracle.ew_cfg4(A, B, C, threads=threads)
    d = np.float32(1) + _expf(-B)
    t = (A + B) * C - A
    ref = np.where(t > 0, t, np.float32(0)) / d
    assert np.array_equal(out, ref)  # values; a ReLU zero may carry either sign


@settings(max_examples=40, deadline=None)
@given(Bn=st.integers(1, 64), C=st.integers(2, 12), seed=st.integers(0, 2 ** 31 - 1))
def test_softmax_ce_textbook_order(Bn, C, seed):
    """The textbook softmax cross-entropy in the order the kernels use (max, sum of expf(z - m)
    c ascending, lse = m + logf(s), loss summed i ascending times 1/B; dz = (expf(z - lse) -
    onehot) * (1/B)) with libm's expf / logf: bit-exact."""
    rng = np.random.default_rng(seed)
    z = _rand(rng, (Bn, C), 3.0)
    y = rng.integers(0, C, Bn).astype(np.int32)
    loss, dz = oracle.softmax_ce(z, y)
    invB = np.float32(1) / np.float32(Bn)
    total = np.float32(0)
    dz_ref = np.empty_like(z)
    for i in range(Bn):
        m = z[i].max()
        s = np.float32(0)
        for c in range(C):
            s = np.float32(s + _libm.expf(np.float32(z[i, c] - m)))
        lse = np.float32(m + np.float32(_libm.logf(s)))
        total = np.float32(total + np.float32(lse - z[i, y[i]]))
        for c in range(C):
            p = np.float32(_libm.expf(np.float32(z[i, c] - lse)))
            dz_ref[i, c] = np.float32(np.float32(p - (1 if c == y[i] else 0)) * invB)
    assert np.float32(loss) == np.float32(total * invB)
    assert _bits_equal(dz, dz_ref)


@settings(max_examples=40, deadline=None)
@given(S=st.integers(1, 96), D=st.sampled_from([8, 16, 64, 128]), causal=st.booleans(),
       seed=st.integers(0, 2 ** 31 - 1))
def test_attention_rows_against_float64(S, D, causal, seed):
    """The textbook attention the FlashAttention kernel is checked against (no reference code,
    parity unpinned): O = softmax(scale * Q K^T + causal mask) V and LSE = m + log(sum), here
    against a float64 numpy evaluation (relative error of O <= 1e-5, LSE <= 1e-5 absolute)."""
    rng = np.random.default_rng(seed)
    q, k, v = (_rand(rng, (S, D)) for _ in range(3))
    scale = 1.0 / np.sqrt(D)
    o, lse = oracle.attention_rows(q, k, v, scale, causal)
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    if causal:
        s = np.where(np.tril(np.ones((S, S), bool)), s, -np.inf)
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=1, keepdims=True)
    o_ref = (p / l) @ v.astype(np.float64)
    lse_ref = (m + np.log(l))[:, 0]
    assert np.abs(o - o_ref).max() <= 1e-5 * max(np.abs(o_ref).max(), 1.0)
    assert np.abs(lse - lse_ref).max() <= 1e-5 * max(np.abs(lse_ref).max(), 1.0)
