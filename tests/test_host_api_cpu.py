"""Runs the C++ host-API tests (tests/cpp/test_host_api.cpp) that need no GPU: known answers
of the rolling hash / region key / cost model derived from the reference code, registry
install-preemption-fallback semantics, graph lowering, hot-path trigger, backward keys."""
import os
import subprocess

import pytest

from tests.cpp.build import build, build_tsan


def test_host_api_cpu():
    exe = build()
    r = subprocess.run([str(exe), "--cpu"], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout


def test_registries_concurrency_under_thread_sanitizer():
    """The concurrency tests (dispatch threads against a compile thread installing and
    reinstalling kernels; dispatch threads recording into the hot-path manager while its
    background compiles install regions; autograd threads recording backward sequences while
    fused-backward compiles run) with the host mirror built under ThreadSanitizer: any data
    race in the registries, the manager or the backward capture fails them."""
    exe = build_tsan()
    if exe is None:
        pytest.skip("g++ -fsanitize=thread unavailable")
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1 exitcode=66 second_deadlock_stack=1")
    for name in ("registries_concurrent_install_and_dispatch", "hot_path_concurrent_record_and_compile",
                 "backward_capture_concurrent_recording"):
        r = subprocess.run([str(exe), "--cpu", "--only", name], capture_output=True, text=True, timeout=600,
                           env=env)
        print(r.stdout)
        assert "ThreadSanitizer" not in r.stderr, r.stderr[-4000:]
        assert r.returncode == 0, r.stdout + r.stderr[-4000:]
        assert "1 tests" in r.stdout and "0 failures" in r.stdout
