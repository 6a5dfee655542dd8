"""Sanitizer builds of the host runtime (no GPU, no Python bindings).

csrc/tests/runtime_stress.cpp drives the scheduler (random requests, aborts,
failed steps, every victim policy, swap slots, long-context policies), the
CacheMesh tiers, the JSON Schema matcher (fuzzed bytes and mask/feed
agreement) and the worker pool.  It is compiled here twice:

  * AddressSanitizer + UndefinedBehaviorSanitizer over everything
    (heap overflows, use-after-free, leaks, signed overflow, bad shifts);
  * ThreadSanitizer over the worker pool (data races in job publication,
    the spin-then-sleep hand-off and the completion count).

A sanitizer report or a failed invariant makes the binary exit non-zero.
The reference has no sanitizer runs (its safety rests on Rust ownership and
mutex-poison recovery, e.g. crates/engine/src/lib.rs:3); the runtime here is
C++, so the compiler sanitizers stand in for the borrow checker.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCES = ["csrc/tests/runtime_stress.cpp", "csrc/runtime/scheduler.cpp", "csrc/runtime/block_manager.cpp",
           "csrc/runtime/cachemesh.cpp", "csrc/runtime/schema_matcher.cpp", "csrc/runtime/thread_pool.cpp"]
REPORTS = ("AddressSanitizer", "LeakSanitizer", "runtime error:", "ThreadSanitizer", "CHECK failed")


def _build_and_run(flags, args, tmp):
    exe = os.path.join(tmp, "stress")
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fno-omit-frame-pointer", "-DBLOOM_NO_PYTHON", *flags,
           "-Icsrc/runtime", *SOURCES, "-o", exe, "-lpthread"]
    b = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    if b.returncode != 0 and "sanitizer" in b.stderr.lower() and "cannot find" in b.stderr.lower():
        pytest.skip("sanitizer runtime library not installed: " + b.stderr[-300:])
    assert b.returncode == 0, b.stderr[-3000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0:exitcode=41",
               UBSAN_OPTIONS="print_stacktrace=1:halt_on_error=1:exitcode=42",
               TSAN_OPTIONS="halt_on_error=1:exitcode=43")
    r = subprocess.run([exe, *args], capture_output=True, text=True, timeout=600, env=env)
    return r


@pytest.fixture
def tmpdir_path():
    d = tempfile.mkdtemp(prefix="bloom-san-")
    yield d
    shutil.rmtree(d, ignore_errors=True)


@pytest.mark.skipif(shutil.which("g++") is None, reason="no host C++ compiler")
def test_runtime_under_asan_ubsan(tmpdir_path):
    r = _build_and_run(["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"], [], tmpdir_path)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert "runtime stress ok" in r.stdout
    assert not any(k in out for k in REPORTS), out[-4000:]


@pytest.mark.skipif(shutil.which("g++") is None, reason="no host C++ compiler")
def test_thread_pool_under_tsan(tmpdir_path):
    r = _build_and_run(["-fsanitize=thread"], ["pool"], tmpdir_path)
    out = r.stdout + r.stderr
    if "FATAL: ThreadSanitizer: unexpected memory mapping" in out:
        pytest.skip("ThreadSanitizer cannot map its shadow memory on this kernel")
    assert r.returncode == 0, out[-4000:]
    assert not any(k in out for k in REPORTS), out[-4000:]
