"""Runs the C++ host-API tests (tests/cpp/test_host_api.cpp) that need no GPU: known answers
of the rolling hash / region key / cost model derived from the reference code, registry
install-preemption-fallback semantics, graph lowering, hot-path trigger, backward keys."""
import os
import subprocess

import pytest

from tests.cpp.build import build, build_sanitized, build_tsan


def test_host_api_cpu():
    exe = build()
    r = subprocess.run([str(exe), "--cpu"], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout


def test_host_api_under_thread_sanitizer():
    """Every CPU test of the host API with the host mirror built under ThreadSanitizer,
    including the three concurrency tests:
    - dispatch threads against a compile thread installing and reinstalling kernels;
    - dispatch threads recording into the hot-path manager while its background compiles
      install regions;
    - autograd threads recording backward sequences while fused-backward compiles run.
    Any data race in the registries, the engine, the manager or the backward capture fails it."""
    exe = build_tsan()
    if exe is None:
        pytest.skip("g++ -fsanitize=thread unavailable")
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1 exitcode=66 second_deadlock_stack=1")
    r = subprocess.run([str(exe), "--cpu"], capture_output=True, text=True, timeout=900, env=env)
    print(r.stdout)
    assert "ThreadSanitizer" not in r.stderr, r.stderr[-4000:]
    assert r.returncode == 0, r.stdout + r.stderr[-4000:]
    assert "0 failures" in r.stdout
    for name in ("registries_concurrent_install_and_dispatch", "hot_path_concurrent_record_and_compile",
                 "backward_capture_concurrent_recording"):
        assert f"PASS {name}" in r.stdout


def test_host_api_under_address_and_ub_sanitizers():
    """Every CPU test of the host API with the host mirror built under AddressSanitizer and
    UndefinedBehaviorSanitizer (leak checking on): no memory error, leak or undefined behaviour
    in the registries, engine, hot-path manager, backward capture or tensor shim."""
    exe = build_sanitized("address,undefined")
    if exe is None:
        pytest.skip("g++ -fsanitize=address,undefined unavailable")
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:halt_on_error=1",
               UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")
    r = subprocess.run([str(exe), "--cpu"], capture_output=True, text=True, timeout=900, env=env)
    print(r.stdout)
    for marker in ("AddressSanitizer", "LeakSanitizer", "runtime error"):
        assert marker not in r.stderr, r.stderr[-4000:]
    assert r.returncode == 0, r.stdout + r.stderr[-4000:]
    assert "0 failures" in r.stdout
