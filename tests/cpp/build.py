"""Build tests/cpp/native_tests against the C++ API (libstream_runtime.so) and
the CPU oracle. Output: tests/cpp/_build/native_tests (git-ignored)."""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "_build" / "native_tests"


def build(force: bool = False) -> Path:
    lib = ROOT / "streaming_transformer_b200" / "lib"
    oracle = ROOT / "oracle" / "_build"
    src = HERE / "native_tests.cpp"
    deps = [src, lib / "libstream_runtime.so", oracle / "libst_oracle.so", *sorted((ROOT / "include").glob("*"))]
    if not force and OUT.exists() and all(d.exists() and d.stat().st_mtime <= OUT.stat().st_mtime for d in deps):
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    cxx = shutil.which("g++") or "g++"
    cmd = [cxx, "-O1", "-std=c++20", "-I", str(ROOT / "include"), "-I", str(ROOT / "oracle"), "-o", str(OUT),
           str(src), "-L", str(lib), "-lstream_runtime", "-lstreaming_b200", "-L", str(oracle), "-lst_oracle",
           f"-Wl,-rpath,{lib}", f"-Wl,-rpath,{oracle}", "-Wl,-rpath,$ORIGIN/../../../streaming_transformer_b200/lib",
           "-Wl,-rpath,$ORIGIN/../../../oracle/_build"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("native_tests build failed")
    return OUT


if __name__ == "__main__":
    print(build("--force" in sys.argv))
