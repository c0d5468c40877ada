"""CPU-only checks of the C ABI library: it loads without a GPU driver, exports every
function that include/*.h declares, and reports (rather than crashes on) a missing device."""
import ctypes

import pytest

from c3_b200 import _lib


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _lib.declared_symbols()
    assert "c3cu_linear_bias_relu_fwd" in declared
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, f"declared in include/*.h but not exported: {missing}"


def test_version_and_status_calls_without_gpu():
    import torch
    lib = _lib.load()
    assert lib.c3cu_version() >= 1
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; the no-device path is not reachable")
    assert lib.c3cu_device_check() == -5  # C3CU_ERR_UNSUPPORTED
    assert "device" in _lib.last_error().lower()
    # entry points refuse cleanly before touching memory
    rc = lib.c3cu_linear_bias_relu_fwd(None, None, None, None, None, 1, 1, 1, 0, None)
    assert rc == -5


def test_collective_cluster_setter_checks_its_value():
    lib = _lib.load()
    try:
        assert lib.c3cu_set_collective_cluster(2) == 0
        assert lib.c3cu_set_collective_cluster(3) == -1
        assert "1 or 2" in _lib.last_error()
        assert lib.c3cu_set_collective_cluster(0) == -1
    finally:
        assert lib.c3cu_set_collective_cluster(1) == 0


def test_workspace_size_queries_are_pure_host():
    lib = _lib.load()
    assert lib.c3cu_relu_mask_db_workspace(16384, 4096) >= 32 * 4096 * 4
    assert lib.c3cu_relu_mask_db_workspace(0, 10) > 0
    assert lib.c3cu_sum_rows_f32_workspace(5, 5) > 0


def test_device_wrapper_passes_host_calls_through():
    """on_tensor_device leaves calls without CUDA tensors alone (no device is touched)."""
    import torch
    from c3_b200 import _lib

    @_lib.on_tensor_device
    def f(a, b=None, xs=()):
        return a.sum() + (0 if b is None else b.sum()) + sum(x.sum() for x in xs)

    t = torch.ones(3)
    assert float(f(t, b=t, xs=[t, t])) == 12.0


def _header_prototypes():
    """{name: (return type, [parameter types])} of every function declared in include/*.h."""
    import re
    from pathlib import Path
    protos = {}
    for h in sorted((Path(_lib.PKG).parent / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"#[^\n]*", "", text)
        for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(c3cu_\w+)\s*\(([^)]*)\)\s*;", text):
            ret, name, params = m.group(1).strip(), m.group(2), m.group(3).strip()
            plist = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
            types = [re.sub(r"\s*\b\w+$", "", p) if not p.endswith("*") else p for p in plist]
            protos[name] = (ret, types)
    return protos


def _kind_of_c(t: str) -> str:
    t = t.replace("const", "").strip()
    if "*" in t or t in ("c3cu_stream_t",):
        return "ptr"
    if t == "float":
        return "f32"
    if t == "double":
        return "f64"
    if t in ("int", "int32_t", "uint32_t", "unsigned", "unsigned int"):
        return "i32"
    if t in ("int64_t", "size_t", "uint64_t", "long long"):
        return "i64"
    return "?" + t


def _kind_of_ctypes(t) -> str:
    if t in (ctypes.c_void_p, ctypes.c_char_p) or (isinstance(t, type) and issubclass(t, ctypes._Pointer)):
        return "ptr"
    if t is ctypes.c_float:
        return "f32"
    if t is ctypes.c_double:
        return "f64"
    if t in (ctypes.c_int, ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint):
        return "i32"
    if t in (ctypes.c_int64, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_longlong):
        return "i64"
    return "?" + repr(t)


def test_ctypes_signatures_match_the_header():
    """Every signature the Python wrappers declare agrees with include/c3cu.h in arity and in
    the kind of each argument and of the result: a wrong one would pass a stream or a size in
    the wrong slot without any error."""
    protos = _header_prototypes()
    assert "c3cu_gemm_bf16" in protos and len(protos["c3cu_gemm_bf16"][1]) == 16
    bad = []
    for name, (args, res) in _lib._SIGNATURES.items():
        assert name in protos, f"{name} has a ctypes signature but no declaration"
        ret, ptypes = protos[name]
        want = [_kind_of_c(t) for t in ptypes]
        got = [_kind_of_ctypes(t) for t in args]
        if want != got:
            bad.append(f"{name}: header {want} vs ctypes {got}")
        if _kind_of_c(ret) != _kind_of_ctypes(res):
            bad.append(f"{name}: returns {ret} in the header, {res} in ctypes")
    assert not bad, "\n".join(bad)
