"""The C++ engine core (scheduler, block manager, sampling oracle, n-gram
speculator, request queue) under AddressSanitizer + UndefinedBehaviorSanitizer:
tests/cpp/core_fuzz.cpp drives randomised workloads with preemption, forks,
speculative appends and aborts, and checks batch invariants."""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CORE = os.path.join(ROOT, "swiftllm_b200", "csrc", "core")


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_core_fuzz_asan_ubsan(tmp_path):
    exe = str(tmp_path / "core_fuzz")
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined",
           "-fno-sanitize-recover=undefined", f"-I{CORE}",
           os.path.join(ROOT, "tests", "cpp", "core_fuzz.cpp"),
           os.path.join(CORE, "scheduler.cpp"), os.path.join(CORE, "block_manager.cpp"),
           os.path.join(CORE, "sampler.cpp"), "-o", exe, "-lpthread"]
    b = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    if b.returncode != 0 and "asan" in b.stderr.lower():
        pytest.skip("sanitizer runtime not available: " + b.stderr[-300:])
    assert b.returncode == 0, b.stderr[-3000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0",
               UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0 and "CORE_FUZZ_OK" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])
