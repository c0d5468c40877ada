"""The Python wrappers check every operand and caller-supplied output (shape, dtype, layout)
before any C call: the C ABI takes bare pointers, so a size that disagrees with an allocation
would make a kernel or a TMA descriptor reach past it. Run on CPU tensors with the library
replaced by a stub that fails the test if any entry point is reached."""
from __future__ import annotations

import pytest
import torch

import c3_b200
from c3_b200 import _lib, attention, elementwise, exact, linear
from c3_b200._lib import C3CUError


class _NoCalls:
    def __getattr__(self, name):
        raise AssertionError(f"{name} was reached although an operand check should have refused")


@pytest.fixture(autouse=True)
def no_library(monkeypatch):
    monkeypatch.setattr(_lib, "load", lambda *a, **k: _NoCalls())


@pytest.fixture
def any_device(monkeypatch):
    """Lets CPU tensors pass the device check, so that each shape check is reached; a call that
    got past every check would then hit the stub library and fail the test."""
    monkeypatch.setattr(linear, "_device_ok", lambda t: True)


bf16, f32, i32 = torch.bfloat16, torch.float32, torch.int32


def z(*shape, dtype=bf16):
    return torch.zeros(shape, dtype=dtype)


def refused(fn, *args, match: str = "", **kwargs):
    with pytest.raises(C3CUError) as e:
        fn(*args, **kwargs)
    assert e.value.code == -1
    if match:
        assert match in str(e.value), str(e.value)
    return str(e.value)


M, N, K = 64, 96, 32
MW = (N + 31) // 32


def test_forward_operands_and_outputs(any_device):
    X, W, b = z(M, K), z(N, K), z(N, dtype=f32)
    refused(linear.forward, X, z(N, K + 8), b, match="expected shape")          # W's K disagrees
    refused(linear.forward, X, W, z(N - 1, dtype=f32), match="expected shape")  # b too short
    refused(linear.forward, X, z(K + 8, N), b, "kn", match="expected shape")
    refused(linear.forward, X, W, b, Y=z(M, N - 8), match="expected shape")
    refused(linear.forward, X, W, b, Y=z(M, N, dtype=f32), match="bfloat16")
    refused(linear.forward, X, W, b, mask=z(M, MW - 1, dtype=i32), match="expected shape")
    refused(linear.forward, X, W, b, mask=z(M + 1, MW, dtype=i32), match="expected shape")
    refused(linear.forward, X.t(), W, b, match="contiguous")


def test_relu_mask_db_operands_and_outputs(any_device):
    dY, mask = z(M, N), z(M, MW, dtype=i32)
    refused(linear.relu_mask_db, dY, z(M, MW + 1, dtype=i32), match="expected shape")
    refused(linear.relu_mask_db, dY, z(M - 1, MW, dtype=i32), match="expected shape")
    refused(linear.relu_mask_db, dY, mask, dZ=z(M, N - 1), match="expected shape")
    refused(linear.relu_mask_db, dY, mask, db=z(N + 1, dtype=f32), match="expected shape")
    refused(linear.relu_mask_db, dY, mask, db=z(N, dtype=bf16), match="float32")


def test_grad_input_checks_weight_against_dz(any_device):
    dZ = z(M, N)
    refused(linear.grad_input, dZ, z(N + 8, K), match="expected shape")       # W's N disagrees
    refused(linear.grad_input, dZ, z(K, N + 8), "kn", match="expected shape")
    refused(linear.grad_input, dZ, z(N, K), dX=z(M, K + 8), match="expected shape")


def test_grad_weight_checks_rows_and_output(any_device):
    dZ, X = z(M, N), z(M, K)
    refused(linear.grad_weight, dZ, z(M + 1, K), match="expected shape")     # X's rows disagree
    refused(linear.grad_weight, dZ, X, dW=z(K, N, dtype=f32), match="expected shape")
    refused(linear.grad_weight, dZ, X, "kn", dW=z(N, K, dtype=f32), match="expected shape")
    refused(linear.grad_weight, dZ, X, dW=z(N, K, dtype=torch.float16), match="float32 or bfloat16")
    refused(linear.grad_weight, dZ, X, dW=z(N, K + 8, dtype=f32)[:, :K], match="contiguous")


def test_general_gemm_checks_majors_sizes_and_epilogue_operands(any_device):
    A, B = z(M, K), z(N, K)
    refused(linear.gemm, A, B, False, False, _lib.EPI_STORE_BF16, z(M, N), M=M + 1, match="expected shape")
    refused(linear.gemm, A, B, False, False, _lib.EPI_STORE_BF16, z(M, N), K=K + 8, match="expected shape")
    refused(linear.gemm, A, B, True, False, _lib.EPI_STORE_BF16, z(K, N), match="expected shape")
    refused(linear.gemm, A, B, False, False, _lib.EPI_STORE_F32, z(M, N), match="float32")
    refused(linear.gemm, A, B, False, False, _lib.EPI_STORE_BF16, z(M, N - 8), match="expected shape")
    refused(linear.gemm, A, B, False, False, _lib.EPI_BIAS_STORE_F32, z(M, N, dtype=f32), match="bias")
    refused(linear.gemm, A, B, False, False, _lib.EPI_BIAS_STORE_F32, z(M, N, dtype=f32),
            bias=z(N - 1, dtype=f32), match="expected shape")
    refused(linear.gemm, A, B, False, False, _lib.EPI_BIAS_RELU_MASK, z(M, N), bias=z(N, dtype=f32),
            match="mask")
    refused(linear.gemm, A, B, False, False, _lib.EPI_BIAS_RELU_MASK, z(M, N), bias=z(N, dtype=f32),
            mask=z(M, MW - 1, dtype=i32), match="expected shape")
    refused(linear.gemm, A, B, False, False, 9, z(M, N), match="epilogue")
    wide = z(K, 2 * M)
    refused(linear.gemm, wide[:, :M].t(), B, False, False, _lib.EPI_STORE_BF16, z(M, N),
            match="stride")


def test_elementwise_checks_counts(any_device):
    A = z(1000, dtype=f32)
    refused(elementwise.chain_cfg4, A, z(999, dtype=f32), A, match="1000 elements")
    refused(elementwise.chain_cfg4, A, A, A, out=z(999, dtype=f32), match="1000 elements")
    refused(elementwise.chain_cfg4, A, A, z(1000, dtype=bf16), match="fp32")
    refused(elementwise.program, [A], [(1, 0, 0, 1)], [], 1, 2000, out=z(1000, dtype=f32),
            match="writes 2000")
    refused(elementwise.program, [z(0, dtype=f32)], [(1, 0, 0, 1)], [], 1, 10, match="at least one")
    refused(elementwise.sum_rows, z(8, 16, dtype=f32), out=z(15, dtype=f32), match="expected shape")
    refused(elementwise.backward_chain, ["ReLU"], A, [z(999, dtype=f32)], match="1000 elements")
    refused(elementwise.backward_chain, ["ReLU", "Tanh"], A, [A], match="saved inputs")
    refused(elementwise.backward_chain, ["ReLU"], A, [A], outs=[z(10, dtype=f32)], match="1000 elements")
    refused(elementwise.backward_chain, ["Cube"], A, [A], match="node types")


def test_attention_checks_shapes(any_device):
    Q = z(1, 2, 256, 128)
    refused(attention.flash_attn_fwd, Q, z(1, 2, 128, 128), Q, match="expected shape")
    refused(attention.flash_attn_fwd, Q, Q, Q, out=z(1, 2, 128, 128), match="expected shape")
    refused(attention.flash_attn_fwd, Q, Q, Q, lse=z(1, 2, 255, dtype=f32), match="expected shape")


def test_exact_checks_inner_dimension_and_bias(any_device):
    A = z(8, 16, dtype=f32)
    refused(exact.matmul, A, z(17, 4, dtype=f32), match="expected shape")
    refused(exact.matmul, A, z(4, 17, dtype=f32), trans_b=True, match="expected shape")
    refused(exact.matmul, A, z(16, 4, dtype=f32), bias=z(3, dtype=f32), match="1 or N=4")
    refused(exact.region_forward, A, z(15, 4, dtype=f32), z(4, dtype=f32), match="expected shape")
    refused(exact.region_forward, A, z(16, 4, dtype=f32), z(0, dtype=f32), match="at least one")


def test_cpu_tensors_refused_before_any_call():
    """Well-formed operands on the CPU are refused for not being on a CUDA device."""
    X, W, b = z(M, K), z(N, K), z(N, dtype=f32)
    refused(linear.forward, X, W, b, match="CUDA")
    refused(linear.relu_mask_db, z(M, N), z(M, MW, dtype=i32), match="CUDA")
    refused(linear.grad_input, z(M, N), W, match="CUDA")
    refused(linear.grad_weight, z(M, N), X, match="CUDA")
    refused(linear.gemm, z(K, 2 * M)[:, :M], W, True, False, _lib.EPI_STORE_BF16, z(M, N), match="CUDA")
    A = z(1000, dtype=f32)
    refused(elementwise.chain_cfg4, A, A, A, match="CUDA")
    Q = z(1, 2, 256, 128)
    refused(attention.flash_attn_fwd, Q, Q, Q, match="CUDA")
    refused(exact.matmul, z(8, 16, dtype=f32), z(16, 4, dtype=f32), match="CUDA")


def test_package_exports_error_type():
    assert c3_b200.C3CUError is C3CUError
