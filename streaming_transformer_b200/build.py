"""Build the native libraries in-tree (sm_100a only).

    python -m streaming_transformer_b200.build [--force]

Outputs (git-ignored, but shipped with the source tree to the GPU box):
    streaming_transformer_b200/lib/libstreaming_b200.so   CUDA kernels + C ABI
    streaming_transformer_b200/lib/libstream_runtime.so   C++ Stream::Runtime / Stream::Model
                                                          API over the C ABI
A target is rebuilt only when one of its sources is newer than it.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = PKG / "host"
LIB = PKG / "lib"
INCLUDE = ROOT / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
# The image exports CC/CXX pointing at a gcc without OpenMP specs; the system
# compiler on PATH is the one nvcc and the C++ layer use.
CXX = shutil.which("g++") or "g++"

GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
              "-ccbin", CXX, *GENCODE]

CUDA_LIB = LIB / "libstreaming_b200.so"
CPP_LIB = LIB / "libstream_runtime.so"


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str], log: Path | None = None) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if log is not None:
        log.write_text(proc.stdout + proc.stderr)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("build failed: " + " ".join(cmd[:3]) + " ...")


def build_cuda(force: bool = False) -> Path:
    units = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "streaming_b200.h"]
    if force or _stale(CUDA_LIB, units + headers):
        LIB.mkdir(exist_ok=True)
        objs = [LIB / (u.stem + ".o") for u in units]
        # Translation units compile in parallel (the flow kernels are the
        # longest); every object is rebuilt because they share the headers.
        procs = [subprocess.Popen([NVCC, *NVCC_FLAGS, "-c", "-o", str(o), str(u)], stdout=subprocess.PIPE,
                                  stderr=subprocess.STDOUT, text=True) for u, o in zip(units, objs)]
        logs, failed = [], False
        for u, p in zip(units, procs):
            out, _ = p.communicate()
            logs.append(f"== {u.name}\n{out}")
            failed |= p.returncode != 0
        (LIB / "ptxas.log").write_text("\n".join(logs))
        if failed:
            sys.stderr.write("\n".join(logs))
            raise RuntimeError("build failed: nvcc -c ...")
        _run([NVCC, *GENCODE, "-shared", "-o", str(CUDA_LIB), *[str(o) for o in objs]])
        for o in objs:
            o.unlink()
    return CUDA_LIB


def build_cpp(force: bool = False) -> Path | None:
    sources = sorted(HOST.glob("*.cpp"))
    if not sources:
        return None
    deps = sources + sorted(INCLUDE.glob("*.hpp")) + [INCLUDE / "streaming_b200.h", CUDA_LIB]
    if force or _stale(CPP_LIB, deps):
        _run([CXX, "-O2", "-std=c++20", "-fPIC", "-shared", "-I", str(INCLUDE), "-o", str(CPP_LIB),
              *[str(s) for s in sources], "-L", str(LIB), "-lstreaming_b200", "-lcrypto",
              "-Wl,-rpath,$ORIGIN"])
    return CPP_LIB


def build(force: bool = False) -> None:
    build_cuda(force)
    build_cpp(force)


if __name__ == "__main__":
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--force", action="store_true")
    a = p.parse_args()
    build(a.force)
    print(CUDA_LIB)
