"""Parity of the tcgen05 Linear+bias+ReLU forward and its captured backward against the
oracle (the reference's fp32 loop arithmetic restated in C), on the same bf16-rounded inputs.

Tolerances: bf16 tensor-core outputs <= 2e-2 relative (normwise and per element with an
rms floor); dZ (mask apply) bit-exact; ReLU mask bit-exact against the kernel's own
pre-activation (mask == (Y > 0)), and against the oracle's fp32 pre-activation except for
sign flips at |z| below the accumulation-order error."""
import numpy as np
import pytest
import torch

import oracle
from c3_b200 import linear
from tests.helpers import (TOL_BF16, assert_bf16_close, f32, pack_mask, randn, rel_err,
                           unpack_mask)

pytestmark = pytest.mark.gpu

# (M, N, K): tile-aligned, ragged in every dimension, tiny, the cfg1 layer shapes.
SHAPES = [
    (128, 256, 64),
    (256, 512, 256),
    (200, 264, 136),
    (1, 8, 8),
    (130, 40, 24),
    (300, 520, 1000),
    (128, 256, 784),
    (128, 128, 256),
    (517, 1032, 776),
]


def _fwd_inputs(M, N, K, seed, dev):
    X = randn((M, K), 1.0, seed)
    W = randn((N, K), 1.0 / np.sqrt(K), seed + 1)
    b = randn((N,), 0.1, seed + 2, torch.float32)
    return X.to(dev), W.to(dev), b.to(dev)


def _check_mask(mask_words, Y, z_ref, N):
    bits = unpack_mask(mask_words, N)
    # exact against the kernel's own pre-activation: bit set <=> output > 0
    assert np.array_equal(bits, Y > 0), "mask disagrees with the kernel's own ReLU output"
    flips = bits != (z_ref > 0)
    if flips.any():
        scale = float(np.sqrt(np.mean(z_ref.astype(np.float64) ** 2)))
        worst = float(np.abs(z_ref[flips]).max())
        assert worst <= 1e-3 * scale, f"{int(flips.sum())} mask flips, max |z_ref| {worst:.3e}"
    return int(flips.sum())


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("w_layout", ["nk", "kn"])
def test_forward_parity(cuda_device, M, N, K, w_layout):
    X, W, b = _fwd_inputs(M, N, K, 100 + M + N + K, cuda_device)
    Wl = W if w_layout == "nk" else W.t().contiguous()
    Y, mask = linear.forward(X, Wl, b, w_layout)
    torch.cuda.synchronize()
    out_ref, z_ref = oracle.region_fwd(f32(X), f32(W), f32(b), transB=True)
    assert_bf16_close(f32(Y), out_ref, f"Y[{M},{N},{K}]")
    _check_mask(mask.cpu().numpy().view(np.uint32), f32(Y), z_ref, N)


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("w_layout", ["nk", "kn"])
def test_backward_parity(cuda_device, M, N, K, w_layout):
    seed = 700 + M + N + K
    X = randn((M, K), 1.0, seed).to(cuda_device)
    W = randn((N, K), 1.0 / np.sqrt(K), seed + 1).to(cuda_device)
    dY = randn((M, N), 1e-3, seed + 2).to(cuda_device)
    rng = np.random.default_rng(seed)
    bits = rng.random((M, N)) < 0.5
    mask_np = pack_mask(bits)
    mask = torch.from_numpy(mask_np.view(np.int32)).to(cuda_device)
    Wl = W if w_layout == "nk" else W.t().contiguous()

    dZ, db = linear.relu_mask_db(dY, mask)
    dX = linear.grad_input(dZ, Wl, w_layout)
    dW = linear.grad_weight(dZ, X, w_layout)
    torch.cuda.synchronize()

    dZ_ref = oracle.relu_bwd_mask(f32(dY), mask_np)
    # dZ is a masked copy of bf16 values: bit-exact, signed zeros included
    assert np.array_equal(f32(dZ).view(np.uint32), dZ_ref.view(np.uint32))
    db_ref = oracle.sum_reduce(dZ_ref, axis=0)
    bound = 1e-5 * np.abs(dZ_ref).sum(axis=0) + 1e-12
    assert (np.abs(f32(db) - db_ref) <= bound).all(), "db outside 1e-5 * sum|dZ|"

    dX_ref = oracle.matmul(dZ_ref, f32(W))  # dX = dZ W, W [N, K]
    assert_bf16_close(f32(dX), dX_ref, f"dX[{M},{N},{K}]")
    dW_ref = oracle.matmul(dZ_ref, f32(X), transA=True)  # dW = dZ^T X, [N, K]
    got = f32(dW) if w_layout == "nk" else f32(dW).T
    assert_bf16_close(got, dW_ref, f"dW[{M},{N},{K}]")
    # fp32 output of exact bf16 products: only the summation order differs
    assert rel_err(got, dW_ref) < 1e-4
    # bf16 dW (the data-parallel gradient format): fp32 accumulation, one rounding
    dWb = linear.grad_weight(dZ, X, w_layout, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    gotb = f32(dWb) if w_layout == "nk" else f32(dWb).T
    assert_bf16_close(gotb, dW_ref, f"dW bf16[{M},{N},{K}]")


def test_forward_mask_from_forward_feeds_backward(cuda_device):
    """End to end: the forward's own mask drives the backward (as the captured graph does)."""
    M, N, K = 384, 768, 512
    X, W, b = _fwd_inputs(M, N, K, 5, cuda_device)
    Y, mask = linear.forward(X, W, b)
    dY = randn((M, N), 1e-3, 6).to(cuda_device)
    dX, dW, db = linear.backward(dY, mask, X, W)
    torch.cuda.synchronize()
    _, z_ref = oracle.region_fwd(f32(X), f32(W), f32(b), transB=True)
    dZ_ref = oracle.relu_bwd(f32(dY), z_ref)
    bits = unpack_mask(mask.cpu().numpy().view(np.uint32), N)
    agree = bits == (z_ref > 0)
    # where the kernel's mask agrees with the oracle's sign, the gradients must match
    dZ_k = f32(dY) * bits
    assert np.array_equal(dZ_k[agree], dZ_ref[agree])
    assert_bf16_close(f32(dX), oracle.matmul(dZ_k, f32(W)), "dX e2e")
    assert_bf16_close(f32(dW), oracle.matmul(dZ_k, f32(X), transA=True), "dW e2e")
    assert np.abs(f32(db) - dZ_k.sum(axis=0, dtype=np.float64)).max() <= 1e-5 * np.abs(dZ_k).sum(0).max() + 1e-9


def test_general_gemm_epilogues(cuda_device):
    M, N, K = 200, 300, 160
    A = randn((M, K), 1.0, 11).to(cuda_device)
    B = randn((N, K), 0.1, 12).to(cuda_device)
    bias = randn((N,), 0.5, 13, torch.float32).to(cuda_device)
    ref = f32(A) @ f32(B).T
    out = torch.empty((M, N), dtype=torch.float32, device=cuda_device)
    linear.gemm(A, B, False, False, 3, out, bias=bias, M=M, N=N, K=K)
    out2 = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_device)
    linear.gemm(A, B, False, False, 1, out2, M=M, N=N, K=K)
    torch.cuda.synchronize()
    assert rel_err(f32(out), ref + f32(bias)) < 1e-4
    assert_bf16_close(f32(out2), ref, "store_bf16")


def test_rejects_misaligned_and_bad_shapes(cuda_device):
    from c3_b200 import C3CUError
    X = torch.zeros((16, 12), dtype=torch.bfloat16, device=cuda_device)  # 24-byte rows
    W = torch.zeros((8, 12), dtype=torch.bfloat16, device=cuda_device)
    b = torch.zeros(8, dtype=torch.float32, device=cuda_device)
    with pytest.raises(C3CUError) as e:
        linear.forward(X, W, b)
    assert e.value.code == -2  # C3CU_ERR_ALIGN
    with pytest.raises(C3CUError):
        linear.forward(X[:, :8].contiguous(), W, b[:4].contiguous())


def test_empty_rows(cuda_device):
    X = torch.zeros((0, 64), dtype=torch.bfloat16, device=cuda_device)
    W = torch.zeros((32, 64), dtype=torch.bfloat16, device=cuda_device)
    b = torch.zeros(32, dtype=torch.float32, device=cuda_device)
    Y, mask = linear.forward(X, W, b)
    assert Y.shape == (0, 32) and mask.shape == (0, 1)


@pytest.mark.parametrize("M", [8192])
def test_cfg2_forward_full_size_sampled(cuda_device, M):
    """BASELINE cfg2 at full size: X[8192,4096] N(0,1), W[4096,4096] N(0,0.02), b N(0,0.01).
    Rows are checked against the oracle on a random sample (the oracle is O(N K) per row)."""
    N = K = 4096
    g = torch.Generator(device=cuda_device).manual_seed(2)
    X = torch.randn((M, K), generator=g, device=cuda_device).to(torch.bfloat16)
    W = (torch.randn((N, K), generator=g, device=cuda_device) * 0.02).to(torch.bfloat16)
    b = torch.randn((N,), generator=g, device=cuda_device) * 0.01
    Y, mask = linear.forward(X, W, b)
    torch.cuda.synchronize()
    rows = np.sort(np.random.default_rng(0).choice(M, 24, replace=False))
    rows = np.concatenate([[0, M - 1], rows])
    Xs = f32(X[torch.as_tensor(rows, device=cuda_device)])
    out_ref, z_ref = oracle.region_fwd(Xs, f32(W), f32(b), transB=True, threads=8)
    Ys = f32(Y[torch.as_tensor(rows, device=cuda_device)])
    assert_bf16_close(Ys, out_ref, "cfg2 Y (sampled rows)")
    _check_mask(mask[torch.as_tensor(rows, device=cuda_device)].cpu().numpy().view(np.uint32), Ys, z_ref, N)
    # size-independent property over the whole output: mask == (Y > 0) everywhere
    bits_all = unpack_mask(mask.cpu().numpy().view(np.uint32), N)
    assert np.array_equal(bits_all, f32(Y) > 0)


def test_cfg3_backward_full_size_sampled(cuda_device):
    """BASELINE cfg3 at full size on one GPU: dY[16384,4096] N(0,1e-3), X N(0,1), W N(0,0.02),
    mask from the forward. dX rows and dW rows are checked on random samples; db in full."""
    M, N, K = 16384, 4096, 4096
    g = torch.Generator(device=cuda_device).manual_seed(3)
    X = torch.randn((M, K), generator=g, device=cuda_device).to(torch.bfloat16)
    W = (torch.randn((N, K), generator=g, device=cuda_device) * 0.02).to(torch.bfloat16)
    b = torch.randn((N,), generator=g, device=cuda_device) * 0.01
    dY = (torch.randn((M, N), generator=g, device=cuda_device) * 1e-3).to(torch.bfloat16)
    _, mask = linear.forward(X, W, b)
    dZ, db = linear.relu_mask_db(dY, mask)
    dX = linear.grad_input(dZ, W)
    dW = linear.grad_weight(dZ, X)
    torch.cuda.synchronize()
    # dZ: exact masked copy (checked on the device, whole tensor)
    bits = torch.from_numpy(unpack_mask(mask.cpu().numpy().view(np.uint32), N)).to(cuda_device)
    assert torch.equal(dZ.view(torch.int16), (dY.float() * bits.float()).to(torch.bfloat16).view(torch.int16))
    dZf = f32(dZ)
    db_ref = dZf.sum(axis=0, dtype=np.float64)
    assert (np.abs(f32(db) - db_ref) <= 1e-5 * np.abs(dZf).sum(0) + 1e-12).all()
    rng = np.random.default_rng(1)
    rows = np.sort(rng.choice(M, 16, replace=False))
    dX_ref = oracle.matmul(dZf[rows], f32(W), threads=8)
    assert_bf16_close(f32(dX)[rows], dX_ref, "cfg3 dX (sampled rows)")
    wrows = np.sort(rng.choice(N, 8, replace=False))
    dW_ref = oracle.matmul(np.ascontiguousarray(dZf[:, wrows]), f32(X), transA=True, threads=8)
    assert_bf16_close(f32(dW)[wrows], dW_ref, "cfg3 dW (sampled rows)")


@pytest.fixture
def gemm_variant():
    from c3_b200 import _lib
    L = _lib.load()
    yield lambda v: _lib.check(L.c3cu_set_gemm_variant(v), "c3cu_set_gemm_variant")
    L.c3cu_set_gemm_variant(0)


def test_gemm_cta_cap_keeps_bits_and_is_per_thread(cuda_device, gemm_variant):
    """c3cu_set_gemm_max_ctas (the SMs a DP step leaves to its all-reduce during dX) changes only
    how many clusters share the tiles: with the pair kernel without the split tail (variant 2)
    the results are bit-identical at any cap. The cap belongs to the thread that sets it: a cap of
    2 CTAs (one cluster for 128 tiles, tens of times slower) set on another thread leaves this
    thread's launches at full speed."""
    import threading
    from c3_b200 import _lib
    L = _lib.load()
    gemm_variant(2)
    M, N, K = 2048, 4096, 1024
    X, W, b = _fwd_inputs(M, N, K, 41, cuda_device)
    ref_Y, ref_mask = linear.forward(X, W, b, "nk")

    def timed():
        linear.forward(X, W, b, "nk")  # warm
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        Y, mask = linear.forward(X, W, b, "nk")
        e.record()
        e.synchronize()
        return s.elapsed_time(e), Y, mask

    try:
        t_full, _, _ = timed()
        for cap in (2, 40, 128):
            _lib.check(L.c3cu_set_gemm_max_ctas(cap), "c3cu_set_gemm_max_ctas")
            t, Y, mask = timed()
            assert torch.equal(Y, ref_Y) and torch.equal(mask, ref_mask), f"cap {cap}"
            if cap == 2:
                t_cap2 = t
        _lib.check(L.c3cu_set_gemm_max_ctas(0), "c3cu_set_gemm_max_ctas")
        assert t_cap2 > 8 * t_full, (t_cap2, t_full)  # the cap took effect on this thread
        th = threading.Thread(target=lambda: L.c3cu_set_gemm_max_ctas(2))
        th.start()
        th.join()
        t_other, Y, _ = timed()
        assert torch.equal(Y, ref_Y)
        assert t_other < t_cap2 / 4, (t_other, t_cap2, t_full)  # another thread's cap did not apply
        assert L.c3cu_set_gemm_max_ctas(-1) != 0  # refused
    finally:
        L.c3cu_set_gemm_max_ctas(0)


@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (300, 520, 1000), (517, 1032, 776),
                                   (1024, 768, 4096), (129, 256, 64), (4096, 512, 4096),
                                   (8192, 2560, 4096)])
def test_gemm_variants_agree(cuda_device, gemm_variant, M, N, K):
    """Variant 1 (single-CTA kernel) and variant 2 (CTA-pair kernel) give the same bits: both
    accumulate each output in the same sequential K order. Variant 0 (pair kernel with the
    split-K tail: (4096, 512, 4096) halves every forward and dW tile, (8192, 2560, 4096) the
    forward's last-wave tiles) sums the two K halves of a split tile separately and adds them,
    so its fp32 results differ within the fp32 accumulation error bound (relative to the sum
    of |terms|) and its bf16 results by at most one rounding."""
    X, W, b = _fwd_inputs(M, N, K, 7 + M, cuda_device)
    dY = randn((M, N), 0.01, 8 + M).to(cuda_device)
    outs = {}
    gemm_variant(1)
    _, mask1 = linear.forward(X, W, b, "nk")
    dZ, _ = linear.relu_mask_db(dY, mask1)  # one dZ for every variant: a ReLU-boundary mask
    for v in (1, 2, 0):                     # flip would change dZ by a whole dY element
        gemm_variant(v)
        Y, mask = linear.forward(X, W, b, "nk")
        dX = linear.grad_input(dZ, W, "nk")
        dW = linear.grad_weight(dZ, X, "nk")
        dWb = linear.grad_weight(dZ, X, "nk", out_dtype=torch.bfloat16)
        dWkn = linear.grad_weight(dZ, X, "kn")
        torch.cuda.synchronize()
        outs[v] = [t.cpu() for t in (Y, mask, dX, dW, dWb, dWkn)]
    names = ("Y", "mask", "dX", "dW", "dW_bf16", "dW_kn")
    for name, a, c in zip(names, outs[1], outs[2]):
        assert torch.equal(a, c), f"{name} differs between the kernels at {M}x{N}x{K}"
    Y1, m1, dX1, dW1, dWb1, dWkn1 = outs[1]
    Y0, m0, dX0, dW0, dWb0, dWkn0 = outs[0]
    absprod = (f32(dZ).__abs__().T @ np.abs(f32(X)))  # sum of |terms| of each dW element
    for name, a, c, s_ in (("dW", dW0, dW1, absprod), ("dW_kn", dWkn0, dWkn1, absprod.T)):
        assert ((a - c).abs().numpy() <= 2e-6 * s_ + 1e-30).all(), name
    # bf16 outputs: one rounding of a slightly different fp32 value, so at most one bf16 ulp
    # apart, or both within the fp32 summation error of zero (a ReLU output at the boundary)
    for name, a, c in (("Y", Y0, Y1), ("dX", dX0, dX1), ("dW_bf16", dWb0, dWb1)):
        a, c = a.float(), c.float()
        bound = 2.0 ** -7 * torch.maximum(a.abs(), c.abs()) + 1e-5 * c.abs().max()
        assert ((a - c).abs() <= bound).all(), f"{name}: more than one bf16 ulp"
    # ReLU mask bits can differ only where the pre-activation rounds to about zero
    b0 = unpack_mask(m0.numpy().view(np.uint32), N)
    b1 = unpack_mask(m1.numpy().view(np.uint32), N)
    diff = b0 != b1
    if diff.any():
        y = np.maximum(np.abs(f32(Y0)), np.abs(f32(Y1)))[diff]
        assert y.max() <= 1e-4 * float(np.abs(f32(Y1)).max()), "mask flip away from zero"


def test_tuner_picks_and_applies_a_variant(cuda_device, tmp_path):
    """tune_gemm times the three variants, installs the fastest per shape and persists it; a
    GEMM then runs through the table with the same results as before (within bf16)."""
    from c3_b200 import _lib, tuning
    M, N, K = 1024, 512, 4096
    X, W, b = _fwd_inputs(M, N, K, 5, cuda_device)
    Y0, _ = linear.forward(X, W, b, "nk")
    entries = tuning.tune_gemm([(M, N, K, 0, 0, 0)], iters=3, path=tmp_path / "t.json")
    try:
        (e,) = entries.values()
        assert e["variant"] in (0, 1, 2) and set(e["us"]) == {"0", "1", "2"}
        assert tuning.read(tmp_path / "t.json")["entries"].keys() == entries.keys()
        Y1, _ = linear.forward(X, W, b, "nk")
        torch.cuda.synchronize()
        a, c = f32(Y1), f32(Y0)
        assert (np.abs(a - c) <= 2.0 ** -7 * np.maximum(np.abs(a), np.abs(c)) + 1e-5 * np.abs(c).max()).all()
    finally:
        _lib.load().c3cu_gemm_tune_clear()


def test_prepass_on_two_streams_at_once(cuda_device):
    """Two pre-passes in flight on two streams of one device: each has its own partial-sum
    scratch (per device and stream) and its own strip tickets, so both give the bits of a
    one-stream run."""
    M, N = 8192, 4096
    dY1 = randn((M, N), 0.01, 51).to(cuda_device)
    dY2 = randn((M, N), 0.01, 52).to(cuda_device)
    g = torch.Generator().manual_seed(53)
    m1 = torch.randint(-2 ** 31, 2 ** 31 - 1, (M, N // 32), generator=g, dtype=torch.int32).to(cuda_device)
    m2 = torch.randint(-2 ** 31, 2 ** 31 - 1, (M, N // 32), generator=g, dtype=torch.int32).to(cuda_device)
    r1 = linear.relu_mask_db(dY1, m1)
    r2 = linear.relu_mask_db(dY2, m2)
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    s1.wait_stream(cur)
    s2.wait_stream(cur)
    outs1, outs2 = [], []
    for _ in range(4):
        with torch.cuda.stream(s1):
            outs1.append(linear.relu_mask_db(dY1, m1))
        with torch.cuda.stream(s2):
            outs2.append(linear.relu_mask_db(dY2, m2))
    cur.wait_stream(s1)
    cur.wait_stream(s2)
    torch.cuda.synchronize()
    for (dz, db) in outs1:
        assert torch.equal(dz, r1[0]) and torch.equal(db, r1[1])
    for (dz, db) in outs2:
        assert torch.equal(dz, r2[0]) and torch.equal(db, r2[1])


def test_fused_dw_allreduce_single_rank_is_the_dw_gemm(cuda_device):
    """c3cu_gemm_dw_allreduce with world = 1 has nothing to sum: it is the bf16 dW GEMM (same
    bits as grad_weight's), and it refuses a multi-rank call whose buffers are not set."""
    import ctypes

    from c3_b200 import _lib
    L = _lib.load()
    M, N, K = 640, 384, 520
    dZ = randn((M, N), 1e-2, 41).to(cuda_device)
    X = randn((M, K), 1.0, 42).to(cuda_device)
    dW = torch.empty((N, K), dtype=torch.bfloat16, device=cuda_device)
    s = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    rc = L.c3cu_gemm_dw_allreduce(ctypes.c_void_p(dZ.data_ptr()), ctypes.c_void_p(X.data_ptr()),
                                  ctypes.c_void_p(dW.data_ptr()), None, None, 0, None, None, 0,
                                  M, N, K, 0, 1, 0, s)
    assert rc == 0, _lib.last_error()
    ref = linear.grad_weight(dZ, X, "nk", out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(dW.view(torch.int16), ref.view(torch.int16))
    assert_bf16_close(f32(dW), oracle.matmul(f32(dZ), f32(X), transA=True), "dW (world 1)")
    rc = L.c3cu_gemm_dw_allreduce(ctypes.c_void_p(dZ.data_ptr()), ctypes.c_void_p(X.data_ptr()),
                                  ctypes.c_void_p(dW.data_ptr()), None, None, 0, None, None, 0,
                                  M, N, K, 0, 2, 0, s)
    assert rc == -1 and "null" in _lib.last_error()


def test_split_k_recovers_after_a_partner_wait_runs_out(cuda_device):
    """A split-K tile's second half that gives up waiting for the first half's partial (here:
    the wait limit shortened to 1 ns through c3cu_set_split_wait_ns, no GPU fault) records
    C3CU_ERR_FAULT. The late partner may leave its tile's ticket words set; after the fault is
    read, the next launch clears the split workspace, so the same GEMM is bit-identical again."""
    import ctypes

    from c3_b200 import _lib
    L = _lib.load()
    M, N, K = 16384, 4096, 4096  # dW of cfg3: 256 tiles, the last wave split in K halves
    dZ = randn((M, N), 1e-2, 51).to(cuda_device)
    X = randn((M, K), 1.0, 52).to(cuda_device)
    ref = linear.grad_weight(dZ, X, "nk")
    torch.cuda.synchronize()
    code = ctypes.c_uint32(0)
    faulted = False
    try:
        assert L.c3cu_set_split_wait_ns(1) == 0
        for _ in range(8):
            linear.grad_weight(dZ, X, "nk")
            if L.c3cu_fault_status(ctypes.byref(code)) == -4:  # C3CU_ERR_FAULT, read and cleared
                faulted = True
                break
    finally:
        assert L.c3cu_set_split_wait_ns(0) == 0
    assert faulted, "no split tile's second half ever arrived before its partner published"
    for _ in range(2):
        out = linear.grad_weight(dZ, X, "nk")
        torch.cuda.synchronize()
        assert torch.equal(out, ref)


def test_launch_overlap_keeps_bits(cuda_device):
    """With programmatic dependent launch (c3cu_set_launch_overlap) each GEMM / pre-pass kernel
    may start its prologue while the previous one drains, but waits for it before touching
    memory: the training step's outputs are bit-identical with it on and off."""
    from c3_b200 import _lib
    L = _lib.load()
    M, N, K = 2048, 1024, 768
    X = randn((M, K), 1.0, 61).to(cuda_device)
    W = randn((N, K), 0.05, 62).to(cuda_device)
    b = randn((N,), 0.05, 63, torch.float32).to(cuda_device)
    dY = randn((M, N), 1e-2, 64).to(cuda_device)

    def step():
        Y, mask = linear.forward(X, W, b)
        dZ, db = linear.relu_mask_db(dY, mask)
        dW = linear.grad_weight(dZ, X, "nk")
        dX = linear.grad_input(dZ, W, "nk")
        return Y, mask, dZ, db, dW, dX

    ref = step()
    torch.cuda.synchronize()
    try:
        assert L.c3cu_set_launch_overlap(1) == 0
        for _ in range(3):
            got = step()
        torch.cuda.synchronize()
    finally:
        assert L.c3cu_set_launch_overlap(0) == 0
    for r, g in zip(ref, got):
        assert torch.equal(r, g)
