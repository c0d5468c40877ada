"""Parity of the single-pass elementwise kernels against the oracle (fp32: <= 1e-5 relative)."""
import numpy as np
import pytest
import torch

import oracle
from c3_b200 import elementwise as ew
from tests.helpers import TOL_F32

pytestmark = pytest.mark.gpu


def _cfg4_inputs(n, seed, dev):
    g = torch.Generator().manual_seed(seed)
    A = torch.rand(n, generator=g) * 8 - 4
    B = torch.rand(n, generator=g) * 16 - 8
    C = torch.rand(n, generator=g) * 8 - 4
    return A.to(dev), B.to(dev), C.to(dev)


def _assert_f32_close(out, ref, what, tol=TOL_F32, atol=0.0):
    """Per element |out - ref| <= tol * |ref| + atol; NaN where the oracle has NaN.
    atol is the conditioning floor of programs that cancel (sum of terms of opposite sign):
    a few ulp of the largest intermediate term."""
    assert np.array_equal(np.isnan(out), np.isnan(ref)), f"{what}: NaN pattern differs"
    both_nan = np.isnan(out) & np.isnan(ref)
    o, r = out[~both_nan], ref[~both_nan]
    err = np.abs(o - r)
    bad = err > tol * np.abs(r) + atol
    assert not bad.any(), f"{what}: {int(bad.sum())} elements, max rel {(err / np.maximum(np.abs(r), 1e-30)).max():.3e}"


@pytest.mark.parametrize("n", [0, 1, 3, 4, 5, 1023, 4096, 1 << 20, (1 << 20) + 7])
def test_chain_cfg4_small(cuda_device, n):
    A, B, C = _cfg4_inputs(n, 40 + n % 97, cuda_device)
    out = ew.chain_cfg4(A, B, C)
    torch.cuda.synchronize()
    ref = oracle.ew_cfg4(A.cpu().numpy(), B.cpu().numpy(), C.cpu().numpy())
    _assert_f32_close(out.cpu().numpy(), ref, f"cfg4 n={n}")


def test_chain_cfg4_unaligned_views(cuda_device):
    n = 100003
    A, B, C = _cfg4_inputs(n + 1, 7, cuda_device)
    A1, B1, C1 = A[1:], B[1:], C[1:]  # 4-byte offset: forces the scalar path
    out = torch.empty(n + 1, device=cuda_device)[1:]
    ew.chain_cfg4(A1, B1, C1, out)
    torch.cuda.synchronize()
    ref = oracle.ew_cfg4(A1.cpu().numpy(), B1.cpu().numpy(), C1.cpu().numpy())
    _assert_f32_close(out.cpu().numpy(), ref, "cfg4 unaligned")


def test_chain_cfg4_full_size(cuda_device):
    """BASELINE cfg4 at full size (2^28 elements); the oracle runs on 8 threads."""
    n = 1 << 28
    g = torch.Generator(device=cuda_device).manual_seed(4)
    A = torch.rand(n, generator=g, device=cuda_device) * 8 - 4
    B = torch.rand(n, generator=g, device=cuda_device) * 16 - 8
    C = torch.rand(n, generator=g, device=cuda_device) * 8 - 4
    out = ew.chain_cfg4(A, B, C)
    torch.cuda.synchronize()
    ref = oracle.ew_cfg4(A.cpu().numpy(), B.cpu().numpy(), C.cpu().numpy(), threads=8)
    _assert_f32_close(out.cpu().numpy(), ref, "cfg4 full size")


PROGRAMS = {
    # relu((a + b) * c - a) / (1 + exp(-b)) written as a register program
    "cfg4": ([(ew.ADD, 3, 0, 1), (ew.MUL, 3, 3, 2), (ew.SUB, 3, 3, 0), (ew.RELU, 3, 3, 0),
              (ew.NEG, 4, 1, 0), (ew.EXP, 4, 4, 0), (ew.CONST, 5, 0, 0), (ew.ADD, 4, 5, 4),
              (ew.DIV, 3, 3, 4)], [1.0], 3),
    # sigmoid backward chain of the reference: s = 1/(1+exp(-x)); g * s * (1 - s)
    "sigmoid_bwd": ([(ew.SIGMOID, 3, 0, 0), (ew.CONST, 4, 0, 0), (ew.SUB, 4, 4, 3),
                     (ew.MUL, 4, 3, 4), (ew.MUL, 4, 1, 4)], [1.0], 4),
    # tanh via exp (scalar fused path), divide with NaN-on-zero, log, gt; the final add of
    # terms up to 4 in magnitude and opposite signs cancels: absolute floor 4 * 4 ulp(1)
    "mixed": ([(ew.TANH_EXP, 3, 0, 0), (ew.DIV_NANZ, 4, 3, 2), (ew.GT, 5, 0, 1),
               (ew.MUL, 4, 4, 5), (ew.EXP, 6, 1, 0), (ew.LOG, 6, 6, 0), (ew.ADD, 4, 4, 6)], [], 4),
}
PROGRAM_ATOL = {"cfg4": 0.0, "sigmoid_bwd": 0.0, "mixed": 16 * 2.0 ** -23}


@pytest.mark.parametrize("name", list(PROGRAMS))
@pytest.mark.parametrize("n", [1, 5, 4097, 1 << 18])
def test_program_parity(cuda_device, name, n):
    code, consts, out_reg = PROGRAMS[name]
    g = torch.Generator().manual_seed(n)
    a = torch.rand(n, generator=g) * 6 - 3
    b = torch.rand(n, generator=g) * 4 - 2
    c = torch.rand(max(1, n // 1), generator=g) * 4 - 2
    if name == "mixed":
        # The exp-form tanh cancels catastrophically near 0 and a small divisor amplifies
        # that: keep |a| >= 0.5 and |c| >= 0.5 so a 1-ulp expf difference between libms
        # stays within tolerance; exact zeros in c exercise the NaN-on-zero division.
        a = torch.sign(a) * (a.abs() + 0.5)
        c = torch.sign(c) * (c.abs() + 0.5)
        c[::7] = 0.0
    ins = [a, b, c]
    out = ew.program([t.to(cuda_device) for t in ins], code, consts, out_reg, n)
    torch.cuda.synchronize()
    ref = oracle.ew_program([t.numpy() for t in ins], code, consts, out_reg, n)
    _assert_f32_close(out.cpu().numpy(), ref, f"program {name} n={n}", tol=2e-6 * 8,
                      atol=PROGRAM_ATOL[name])


def test_program_broadcast(cuda_device):
    """rhs broadcast by index modulo (RemUI in the reference's scalar loop)."""
    n = 64 * 1000
    x = torch.randn(n)
    bias = torch.randn(64)
    code = [(ew.ADD, 2, 0, 1), (ew.RELU, 2, 2, 0)]
    out = ew.program([x.to(cuda_device), bias.to(cuda_device)], code, [], 2, n)
    torch.cuda.synchronize()
    ref = oracle.ew_program([x.numpy(), bias.numpy()], code, [], 2, n)
    assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("M,N", [(1, 1), (7, 300), (512, 256), (513, 4100), (16384, 4096), (0, 5)])
def test_sum_rows(cuda_device, M, N):
    x = torch.randn((M, N), generator=torch.Generator().manual_seed(M + N))
    out = ew.sum_rows(x.to(cuda_device))
    torch.cuda.synchronize()
    ref = oracle.sum_reduce(x.numpy(), 0) if M > 0 else np.zeros(N, np.float32)
    bound = 1e-5 * np.abs(x.numpy()).sum(axis=0) + 1e-12
    assert (np.abs(out.cpu().numpy() - ref) <= bound).all()
    # deterministic: a second launch on the same workspace gives identical bits
    out2 = ew.sum_rows(x.to(cuda_device))
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), out2.cpu())


CHAINS = [["ReLU", "ReLU"], ["Sigmoid", "Tanh"], ["ReLU", "Sigmoid", "Tanh"], ["Tanh", "Exp", "Log", "Neg"],
          ["Neg", "ReLU", "Neg"], ["Sigmoid", "Sigmoid", "Sigmoid", "Sigmoid"], ["Exp", "Tanh"]]


@pytest.mark.parametrize("types", CHAINS, ids=["+".join(c) for c in CHAINS])
@pytest.mark.parametrize("n", [1, 4097, 1 << 20])
def test_backward_chain_parity(cuda_device, types, n):
    """Fused backward of a unary chain against the oracle's node-by-node gradients: exact for
    ReLU / Neg chains; otherwise within 1e-5 relative plus a floor of 1e-6 of the tensor's
    largest value (1 - s and 1 - t^2 cancel when s or |t| is near 1)."""
    g = torch.Generator().manual_seed(n + len(types))
    grad = torch.randn(n, generator=g)
    xs = []
    for t in types:
        x = torch.randn(n, generator=g) * 2
        if t == "Log":
            x = x.abs() + 0.25
        xs.append(None if t == "Neg" else x)
    outs = ew.backward_chain(types, grad.to(cuda_device), [None if x is None else x.to(cuda_device) for x in xs])
    torch.cuda.synchronize()
    refs = oracle.backward_chain(types, grad.numpy(), [None if x is None else x.numpy() for x in xs])
    exact = all(t in ("ReLU", "Neg") for t in types)
    for k, (o, r) in enumerate(zip(outs, refs)):
        o = o.cpu().numpy()
        if exact:
            assert np.array_equal(o, r), f"node {k}"
        else:
            bound = 1e-5 * np.abs(r) + 1e-6 * np.abs(r).max()
            assert (np.abs(o - r) <= bound).all(), f"node {k}: max err {np.abs(o - r).max():.3e}"


def test_program_multi_output(cuda_device):
    """Two outputs from one pass: (a + b) and (a + b) * c."""
    n = 10000
    a, b, c = (torch.randn(n, generator=torch.Generator().manual_seed(s)) for s in (1, 2, 3))
    import ctypes
    from c3_b200 import _lib
    from c3_b200.linear import _p, _stream
    ins = [t.to(cuda_device) for t in (a, b, c)]
    o1, o2 = torch.empty(n, device=cuda_device), torch.empty(n, device=cuda_device)
    ptrs = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in ins])
    nums = (ctypes.c_int64 * 3)(n, n, n)
    code = bytes([ew.ADD, 3, 0, 1, ew.MUL, 4, 3, 2])
    cbuf = (ctypes.c_uint8 * len(code))(*code)
    regs = (ctypes.c_int * 2)(3, 4)
    outs = (ctypes.c_void_p * 2)(o1.data_ptr(), o2.data_ptr())
    consts = (ctypes.c_float * 1)(0.0)
    rc = _lib.load().c3cu_ew_program_multi(ctypes.cast(ptrs, ctypes.c_void_p), ctypes.cast(nums, ctypes.c_void_p), 3,
                                           ctypes.cast(cbuf, ctypes.c_void_p), 2, ctypes.cast(consts, ctypes.c_void_p),
                                           0, ctypes.cast(regs, ctypes.c_void_p), ctypes.cast(outs, ctypes.c_void_p), 2,
                                           n, _stream(ins[0].device))
    _lib.check(rc, "c3cu_ew_program_multi")
    torch.cuda.synchronize()
    s = (a + b)
    assert torch.equal(o1.cpu(), s)
    assert torch.equal(o2.cpu(), s * c)
