"""Compiles tests/cpp/test_host_api.cpp against the in-tree libc3cu.so and the oracle
(test infrastructure) into tests/cpp/_build/test_host_api."""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
OUT = HERE / "_build" / "test_host_api"


def build() -> Path:
    sys.path.insert(0, str(ROOT))
    from c3_b200 import build as lib_build
    import oracle
    lib = lib_build.build()
    olib = oracle.build()
    src = HERE / "test_host_api.cpp"
    headers = list((ROOT / "c3_b200" / "csrc" / "host").rglob("*.h")) + [ROOT / "include" / "c3cu.h",
                                                                           ROOT / "c3_b200" / "csrc" / "gemm2_schedule.h"]
    if OUT.exists() and all(OUT.stat().st_mtime >= p.stat().st_mtime for p in [src, lib, olib] + headers):
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-pthread", str(src), "-o", str(OUT),
           f"-I{ROOT / 'c3_b200' / 'csrc' / 'host'}", f"-I{ROOT / 'c3_b200' / 'csrc'}", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include",
           f"-L{lib.parent}", "-lc3cu", f"-Wl,-rpath,{lib.parent}", f"-L{olib.parent}", "-loracle",
           f"-Wl,-rpath,{olib.parent}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{' '.join(cmd)}\n{r.stderr}")
    return OUT


DRIVE = HERE / "_build" / "api_drive"


def build_drive() -> Path:
    """tests/cpp/api_drive.cpp: the C3 API driven as a host framework does (the cfg1 training loop
    through the registries, the cfg2 region with host tensors), for the benchmark's API legs."""
    sys.path.insert(0, str(ROOT))
    from c3_b200 import build as lib_build
    import oracle
    lib = lib_build.build()
    olib = oracle.build()
    src = HERE / "api_drive.cpp"
    headers = list((ROOT / "c3_b200" / "csrc" / "host").rglob("*.h")) + [ROOT / "include" / "c3cu.h"]
    if DRIVE.exists() and all(DRIVE.stat().st_mtime >= p.stat().st_mtime for p in [src, lib, olib] + headers):
        return DRIVE
    DRIVE.parent.mkdir(exist_ok=True)
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-pthread", str(src), "-o", str(DRIVE),
           f"-I{ROOT / 'c3_b200' / 'csrc' / 'host'}", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include",
           f"-L{lib.parent}", "-lc3cu", f"-Wl,-rpath,{lib.parent}", f"-L{olib.parent}", "-loracle",
           f"-Wl,-rpath,{olib.parent}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{' '.join(cmd)}\n{r.stderr}")
    return DRIVE


SANITIZERS = {"thread": "test_host_api_tsan", "address,undefined": "test_host_api_asan"}


def build_sanitized(sanitize: str = "thread") -> Path | None:
    """The same test program with the C++ host mirror compiled in under a sanitizer
    (`-fsanitize=thread` for data races; `-fsanitize=address,undefined` for memory errors, leaks
    and undefined behaviour). The C ABI and the oracle come from their libraries as usual (only
    the host sources are instrumented). Sources compile in parallel, then link. Returns None
    when this toolchain cannot build it."""
    import concurrent.futures as cf
    import os
    sys.path.insert(0, str(ROOT))
    from c3_b200 import build as lib_build
    import oracle
    out = HERE / "_build" / SANITIZERS[sanitize]
    objdir = HERE / "_build" / (SANITIZERS[sanitize] + "_obj")
    lib = lib_build.build()
    olib = oracle.build()
    src = HERE / "test_host_api.cpp"
    host = ROOT / "c3_b200" / "csrc" / "host"
    srcs = [src] + sorted(host.rglob("*.cpp"))
    headers = list(host.rglob("*.h")) + [ROOT / "include" / "c3cu.h", ROOT / "c3_b200" / "csrc" / "gemm2_schedule.h"]
    if out.exists() and all(out.stat().st_mtime >= p.stat().st_mtime for p in [lib, olib] + headers + srcs):
        return out
    objdir.mkdir(parents=True, exist_ok=True)
    flags = ["g++", "-std=c++17", "-O1", "-g", f"-fsanitize={sanitize}", "-fno-omit-frame-pointer", "-pthread",
             f"-I{host}", f"-I{ROOT / 'c3_b200' / 'csrc'}", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include"]

    def compile_one(path: Path):
        obj = objdir / (path.relative_to(ROOT).as_posix().replace("/", "_") + ".o")
        r = subprocess.run(flags + ["-c", str(path), "-o", str(obj)], capture_output=True, text=True)
        return obj, r

    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        results = list(ex.map(compile_one, srcs))
    for _, r in results:
        if r.returncode != 0:
            print(f"-fsanitize={sanitize} build unavailable: {r.stderr[-2000:]}")
            return None
    cmd = ["g++", f"-fsanitize={sanitize}", "-pthread"] + [str(o) for o, _ in results] + \
          ["-o", str(out), f"-L{lib.parent}", "-lc3cu", f"-Wl,-rpath,{lib.parent}",
           f"-L{olib.parent}", "-loracle", f"-Wl,-rpath,{olib.parent}", "-L/usr/local/cuda/lib64", "-lcudart",
           "-Wl,-rpath,/usr/local/cuda/lib64"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    shutil.rmtree(objdir, ignore_errors=True)  # intermediates only; the binary's mtime decides rebuilds
    if r.returncode != 0:
        print(f"-fsanitize={sanitize} link failed: {r.stderr[-2000:]}")
        return None
    return out


def build_tsan() -> Path | None:
    return build_sanitized("thread")


if __name__ == "__main__":
    print(build())
