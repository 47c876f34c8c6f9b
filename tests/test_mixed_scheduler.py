"""The mixed prefill/decode scheduler (hllm_b200/adapter/mixed_scheduler.cpp)
on fake backends, on the CPU: tests/cpp/mixed_scheduler_test.cpp, built by
tests/cpp/Makefile against the reference's runtime headers."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BINARY = os.path.join(ROOT, "_build", "mixed_scheduler_test")


def test_mixed_scheduler_on_fake_backends():
    ref = os.environ.get("HLLM_REF_ROOT")
    if not os.path.exists(BINARY) and ref:
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp"), "scheduler",
                        f"REF_ROOT={ref}"], check=False)
    if not os.path.exists(BINARY):
        pytest.skip("scheduler test not built (build() or HLLM_REF_ROOT with the reference tree)")
    r = subprocess.run([BINARY], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "mixed scheduler: ok" in r.stdout
