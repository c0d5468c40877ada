"""Builds libc3cu.so in-tree: every CUDA translation unit for sm_100a plus the C++ host
mirror of the C3 API, linked with the static CUDA runtime so that the library loads on
machines without a GPU driver (calls then report C3CU_ERR_UNSUPPORTED)."""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = CSRC / "host"
OUT_DIR = PKG / "_build"
LIB = PKG / "libc3cu.so"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
            f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{HOST}"] + GENCODE
CXX_FLAGS = ["-std=c++17", "-O2", "-fPIC", "-Wall", "-Wextra", f"-I{ROOT / 'include'}",
             f"-I{HOST}", "-I/usr/local/cuda/include", "-pthread"]


def _sources():
    cu = sorted(CSRC.glob("*.cu"))
    cpp = sorted(CSRC.glob("*.cpp")) + (sorted(HOST.rglob("*.cpp")) if HOST.exists() else [])
    return cu, cpp


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + \
        list((ROOT / "include").glob("*.h")) + list(HOST.rglob("*.h"))
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path) -> Path:
    rel = src.relative_to(PKG).as_posix().replace("/", "_")
    obj = OUT_DIR / (rel + ".o")
    if not _stale(obj, src):
        return obj
    if src.suffix == ".cu":
        cmd = [NVCC] + CU_FLAGS + ["-c", str(src), "-o", str(obj)]
    else:
        cmd = [os.environ.get("CXX", "g++")] + CXX_FLAGS + ["-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj


def build(verbose: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    cu, cpp = _sources()
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(_compile, cu + cpp))
    if LIB.exists() and all(LIB.stat().st_mtime >= o.stat().st_mtime for o in objs):
        return LIB
    cmd = [NVCC, "-shared", "-cudart", "static", "-o", str(LIB)] + [str(o) for o in objs] + \
        GENCODE + ["-Xlinker", "--no-undefined", "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
