"""Build the two native libraries in-tree, into kvsnap_b200/_native/.

    python -m kvsnap_b200.build [--force]

* ``_cuda_native.so``: the pinned pool (csrc/pool.cpp) and the sm_100a
  data-plane kernels (csrc/dataplane.cu), one C ABI (include/kvsnap_cuda.h).
  nvcc ``-gencode arch=compute_100a,code=sm_100a``; the CUDA runtime is linked
  statically, so the library needs only the driver at run time.
* ``_io_native.so``: host CRC32C and the pread/pwrite pool (csrc/io.cpp,
  include/kvsnap_io.h), g++.

A library is rebuilt when any of its sources or headers is newer than it.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
NATIVE = PACKAGE / "_native"
INCLUDE = ROOT / "include"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CUDA_LIB = NATIVE / "_cuda_native.so"
IO_LIB = NATIVE / "_io_native.so"


def _nvcc() -> str:
    found = shutil.which("nvcc") or str(CUDA_HOME / "bin" / "nvcc")
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _stale(target: Path, sources) -> bool:
    if not target.is_file():
        return True
    built = target.stat().st_mtime
    return any(p.stat().st_mtime > built for p in sources)


def _run(cmd):
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode:
        raise RuntimeError(f"build failed: {' '.join(map(str, cmd))}\n{result.stdout}\n{result.stderr}")


def build_cuda(force: bool = False) -> Path:
    sources = [CSRC / "pool.cpp", CSRC / "dataplane.cu"]
    deps = sources + [CSRC / "kvsnap_internal.h", INCLUDE / "kvsnap_cuda.h"]
    if force or _stale(CUDA_LIB, deps):
        NATIVE.mkdir(parents=True, exist_ok=True)
        tmp = CUDA_LIB.with_suffix(".so.tmp")
        _run([_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-Wall", "-cudart", "static", f"-I{INCLUDE}", f"-I{CSRC}",
              *map(str, sources), "-o", str(tmp)])
        os.replace(tmp, CUDA_LIB)
    return CUDA_LIB


def build_io(force: bool = False) -> Path:
    sources = [CSRC / "io.cpp"]
    if force or _stale(IO_LIB, sources + [INCLUDE / "kvsnap_io.h"]):
        NATIVE.mkdir(parents=True, exist_ok=True)
        tmp = IO_LIB.with_suffix(".so.tmp")
        _run([os.environ.get("CXX", "g++"), "-std=c++17", "-O3", "-shared", "-fPIC", "-pthread", "-Wall",
              "-Wextra", "-Werror", f"-I{INCLUDE}", *map(str, sources), "-o", str(tmp)])
        os.replace(tmp, IO_LIB)
    return IO_LIB


def build(force: bool = False) -> None:
    build_io(force)
    build_cuda(force)


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    build(args.force)
    print(CUDA_LIB, IO_LIB)
