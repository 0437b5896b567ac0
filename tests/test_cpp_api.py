"""The C++ drop-in API (include/Runtime.hpp, include/Model.hpp) through the
native test program tests/cpp/native_tests.cpp, which mirrors the reference's
own C++ suites (reference tests/Native.cpp, tests/Lifecycle.cu)."""
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "cpp"))

import build as cpp_build  # noqa: E402


def run_group(group: str):
    exe = cpp_build.build()
    proc = subprocess.run([str(exe), str(ROOT), group], capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    return proc.stdout


def test_cpp_api_without_gpu():
    out = run_group("cpu")
    assert "0 failed" in out


@pytest.mark.gpu
def test_cpp_api_on_gpu():
    out = run_group("gpu")
    assert "0 failed" in out
