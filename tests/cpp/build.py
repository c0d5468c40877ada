"""Compiles tests/cpp/test_host_api.cpp against the in-tree libc3cu.so and the oracle
(test infrastructure) into tests/cpp/_build/test_host_api."""
from __future__ import annotations

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


if __name__ == "__main__":
    print(build())
