"""Loads libc3cu.so (the C-ABI of include/c3cu.h) and declares its signatures.

The product path has no fallback: if the library is missing and cannot be built, or if
the current device is not an sm_100 part, every entry point raises C3CUError."""
from __future__ import annotations

import ctypes
import functools
import re
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libc3cu.so"
HEADERS = [PKG.parent / "include" / "c3cu.h"]

OK = 0
ERR_NAMES = {-1: "INVALID", -2: "ALIGN", -3: "CUDA", -4: "FAULT", -5: "UNSUPPORTED",
             -6: "WORKSPACE"}

W_NK, W_KN = 0, 1
DTYPE_F32, DTYPE_BF16 = 0, 1
EPI_BIAS_RELU_MASK, EPI_STORE_BF16, EPI_STORE_F32, EPI_BIAS_STORE_F32 = 0, 1, 2, 3


class C3CUError(RuntimeError):
    def __init__(self, code: int, where: str, message: str):
        self.code = code
        super().__init__(f"{where}: C3CU_ERR_{ERR_NAMES.get(code, code)} ({code}): {message}")


_lock = threading.Lock()
_lib = None

_vp, _i64, _i, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t

_SIGNATURES = {
    "c3cu_version": ([], _i),
    "c3cu_last_error": ([], ctypes.c_char_p),
    "c3cu_device_check": ([], _i),
    "c3cu_fault_status": ([ctypes.POINTER(ctypes.c_uint32)], _i),
    "c3cu_linear_bias_relu_fwd": ([_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i, _vp], _i),
    "c3cu_relu_mask_db_workspace": ([_i64, _i64], _sz),
    "c3cu_relu_mask_db": ([_vp, _vp, _vp, _vp, _i64, _i64, _vp, _sz, _vp], _i),
    "c3cu_gemm_dx": ([_vp, _vp, _vp, _i64, _i64, _i64, _i, _vp], _i),
    "c3cu_gemm_dw": ([_vp, _vp, _vp, _i64, _i64, _i64, _i, _vp], _i),
    "c3cu_gemm_bf16": ([_vp, _i64, _i, _vp, _i64, _i, _vp, _i64, _i, _vp, _vp, _i64, _i64, _i64,
                        _i64, _vp], _i),
    "c3cu_ew_chain_cfg4": ([_vp, _vp, _vp, _vp, _i64, _vp], _i),
    "c3cu_ew_program": ([_vp, _vp, _i, _vp, _i, _vp, _i, _i, _vp, _i64, _vp], _i),
    "c3cu_sum_rows_f32_workspace": ([_i64, _i64], _sz),
    "c3cu_sum_rows_f32": ([_vp, _vp, _i64, _i64, _vp, _sz, _vp], _i),
    "c3cu_matmul_f32": ([_vp, _vp, _vp, _i64, _i64, _i64, _i, _i, _vp, _i64, _i, _vp], _i),
    "c3cu_region_fwd_f32": ([_vp, _vp, _vp, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _i, _vp], _i),
    "c3cu_sum_rows_f32_exact": ([_vp, _vp, _i64, _i64, _vp], _i),
    "c3cu_matmul_relu_bwd_f32": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i, _i, _vp], _i),
    "c3cu_matmul_colsum_f32": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i, _i, _vp], _i),
    "c3cu_convert": ([_vp, _i, _vp, _i, _i64, _vp], _i),
    "c3cu_set_gemm_max_ctas": ([_i], _i),
    "c3cu_set_collective_cluster": ([_i], _i),
    "c3cu_set_gemm_variant": ([_i], _i),
    "c3cu_set_split_wait_ns": ([ctypes.c_uint64], _i),
    "c3cu_set_launch_overlap": ([_i], _i),
    "c3cu_gemm_tune_set": ([_i64, _i64, _i64, _i, _i, _i, _i], _i),
    "c3cu_gemm_tune_get": ([_i64, _i64, _i64, _i, _i, _i, ctypes.POINTER(_i)], _i),
    "c3cu_gemm_tune_clear": ([], _i),
    "c3cu_nvls_allreduce": ([_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i, _i, ctypes.c_uint32, _i, _vp], _i),
    "c3cu_nvls_allreduce_split": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i, _i, ctypes.c_uint32,
                                   _i, _i, _vp], _i),
    "c3cu_nccl_version": ([ctypes.POINTER(_i)], _i),
    "c3cu_nccl_unique_id": ([_vp], _i),
    "c3cu_nccl_comm_init": ([ctypes.POINTER(_vp), _vp, _i, _i], _i),
    "c3cu_nccl_comm_destroy": ([_vp], _i),
    "c3cu_allreduce_grads": ([_vp, _i64, _i, _vp, _vp], _i),
    "c3cu_gemm_dw_allreduce": ([_vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _i, _i,
                                ctypes.c_uint32, _vp], _i),
    "c3cu_nvls_allreduce_f32": ([_vp, _vp, _vp, _i64, _i64, _i, _i, ctypes.c_uint32, _i, _vp], _i),
    "c3cu_relu_mask_db_noalloc": ([_vp, _vp, _vp, _vp, _i64, _i64, _vp], _i),
    "c3cu_set_attn_variant": ([_i], _i),
    "c3cu_ew_program_multi": ([_vp, _vp, _i, _vp, _i, _vp, _i, _vp, _vp, _i, _i64, _vp], _i),
    "c3cu_ew_backward_chain": ([_vp, _i, _vp, _vp, _vp, _i64, _vp], _i),
    "c3cu_softmax_ce_f32": ([_vp, _vp, _vp, _vp, _i64, _i64, _vp], _i),
    "c3cu_sgd_f32": ([_vp, _vp, _vp, _i, ctypes.c_float, _vp], _i),
    "c3cu_flash_attn_fwd": ([_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_float, _i, _vp], _i),
}


def declared_symbols() -> list[str]:
    """Every function name declared in include/*.h (used by the export test)."""
    names = []
    for h in sorted((PKG.parent / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        names += re.findall(r"\b(c3\w*)\s*\(", text)
    return sorted(set(n for n in names if not n.isupper()))


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            if not build_if_missing:
                raise RuntimeError(f"{LIB_PATH} is missing; build it with `python -m c3_b200.build`")
            from . import build as _build
            _build.build()
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
        return L


def last_error() -> str:
    msg = load().c3cu_last_error()
    return msg.decode() if msg else ""


def check(rc: int, where: str) -> None:
    if rc != OK:
        raise C3CUError(rc, where, last_error())


def device_check() -> None:
    check(load().c3cu_device_check(), "c3cu_device_check")


def fault_status() -> int:
    """Synchronises the device and returns (and clears) the kernels' fault word; raises
    C3CUError(C3CU_ERR_FAULT) when a kernel recorded a fault."""
    code = ctypes.c_uint32(0)
    rc = load().c3cu_fault_status(ctypes.byref(code))
    check(rc, "c3cu_fault_status")
    return code.value


def _cuda_devices(values, found: set) -> None:
    import torch
    for v in values:
        if isinstance(v, torch.Tensor):
            if v.is_cuda:
                found.add(v.device.index)
        elif isinstance(v, (list, tuple)):
            _cuda_devices(v, found)


def on_tensor_device(fn):
    """Runs a wrapper of the C ABI on the device of its CUDA tensor arguments. The library
    launches on the current device with that device's stream, so the call is made with the
    tensors' device current (as torch ops do). Tensors on different devices are refused before
    any launch: a kernel reading another GPU's memory without peer access would fault."""
    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        import torch
        found: set = set()
        _cuda_devices(args, found)
        _cuda_devices(kwargs.values(), found)
        if not found:
            return fn(*args, **kwargs)
        if len(found) > 1:
            raise C3CUError(-1, fn.__name__, f"tensors on different devices: cuda:{sorted(found)}")
        idx = found.pop()
        if idx == torch.cuda.current_device():  # the common case: no device switch
            return fn(*args, **kwargs)
        with torch.cuda.device(idx):
            return fn(*args, **kwargs)
    return wrapper
