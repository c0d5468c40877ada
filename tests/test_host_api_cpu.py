"""Runs the C++ host-API tests (tests/cpp/test_host_api.cpp) that need no GPU: known answers
of the rolling hash / region key / cost model derived from the reference code, registry
install-preemption-fallback semantics, graph lowering, hot-path trigger, backward keys."""
import subprocess

from tests.cpp.build import build


def test_host_api_cpu():
    exe = build()
    r = subprocess.run([str(exe), "--cpu"], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout
