"""Build the two native libraries in-tree, into kvsnap_b200/_native/.

    python -m kvsnap_b200.build [--force]

* ``_cuda_native.so``: the pinned pool (csrc/pool.cpp) and the sm_100a
  data-plane kernels (csrc/dataplane.cu), one C ABI (include/kvsnap_cuda.h).
  nvcc ``-gencode arch=compute_100a,code=sm_100a``; the CUDA runtime is linked
  statically, so the library needs only the driver at run time.
* ``_io_native.so``: host CRC32C and the pread/pwrite pool (csrc/io.cpp,
  include/kvsnap_io.h), g++.

A library is rebuilt unless the stamp beside it (``<library>.stamp``) holds
the SHA-256 of exactly the sources, headers and compiler command it would be
built from now: a prebuilt library from other sources is never reused because
of its timestamp.
"""
from __future__ import annotations

import argparse
import hashlib
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


def _recipe(sources, command) -> str:
    """The SHA-256 of what a library is built from: each input's name and bytes, then the command."""
    digest = hashlib.sha256()
    for path in sources:
        digest.update(path.name.encode() + b"\0" + path.read_bytes() + b"\0")
    digest.update(" ".join(map(str, command)).encode())
    return digest.hexdigest()


def _stamp(target: Path) -> Path:
    return target.with_name(target.name + ".stamp")


def _stale(target: Path, recipe: str) -> bool:
    stamp = _stamp(target)
    return not target.is_file() or not stamp.is_file() or stamp.read_text().strip() != recipe


def _run(cmd):
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode:
        raise RuntimeError(f"build failed: {' '.join(map(str, cmd))}\n{result.stdout}\n{result.stderr}")


def _build(target: Path, sources, deps, compiler, flags, force: bool) -> Path:
    """Compile ``sources`` into ``target`` unless its stamp matches this recipe; then write the stamp."""
    command = [*flags, *map(str, sources)]
    recipe = _recipe(sources + deps, [Path(compiler).name, *command])
    if force or _stale(target, recipe):
        NATIVE.mkdir(parents=True, exist_ok=True)
        tmp = target.with_suffix(".so.tmp")
        _run([compiler, *command, "-o", str(tmp)])
        os.replace(tmp, target)
        _stamp(target).write_text(recipe + "\n")
    return target


def build_cuda(force: bool = False) -> Path:
    flags = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
             "-cudart", "static", f"-I{INCLUDE}", f"-I{CSRC}"]
    return _build(CUDA_LIB, [CSRC / "pool.cpp", CSRC / "dataplane.cu"],
                  [CSRC / "kvsnap_internal.h", INCLUDE / "kvsnap_cuda.h"], _nvcc(), flags, force)


def build_io(force: bool = False) -> Path:
    flags = ["-std=c++17", "-O3", "-shared", "-fPIC", "-pthread", "-Wall", "-Wextra", "-Werror", f"-I{INCLUDE}"]
    return _build(IO_LIB, [CSRC / "io.cpp"], [INCLUDE / "kvsnap_io.h"], os.environ.get("CXX", "g++"), flags, force)


def build(force: bool = False) -> None:
    build_io(force)
    build_cuda(force)


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    build(args.force)
    print(CUDA_LIB, IO_LIB)
