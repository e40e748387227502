"""Build the sm_100a C-ABI library ``loraforge_b200/_lib/liblfb200.so`` with nvcc.

The library is built in-tree so that it travels with the source tree; nothing is
installed into site-packages and no JIT cache is used.  Run ``python -m
loraforge_b200._build`` (or ``__graft_entry__.build()``) after changing a ``.cu``.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
LIBDIR = PACKAGE / "_lib"
LIBRARY = LIBDIR / "liblfb200.so"
SOURCES = ("capi.cu", "grouping.cu", "shrink.cu", "expand.cu", "sgmv.cu", "sgmv_prefill.cu", "base_gemm.cu",
           "peer.cu")
ARCH = ("-gencode", "arch=compute_100a,code=sm_100a")
FLAGS = ("-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr")


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def _digest() -> str:
    h = hashlib.sha256()
    for path in sorted(CSRC.glob("*")) + sorted(INCLUDE.glob("*.h")):
        if path.is_file():
            h.update(path.name.encode())
            h.update(path.read_bytes())
    h.update(repr((ARCH, FLAGS, SOURCES)).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link the shared library."""
    stamp = LIBDIR / "liblfb200.sha256"
    digest = _digest()
    if not force and LIBRARY.exists() and stamp.exists() and stamp.read_text() == digest:
        return LIBRARY
    LIBDIR.mkdir(exist_ok=True)
    build_dir = LIBDIR / "obj"
    build_dir.mkdir(exist_ok=True)
    compiler = nvcc()

    def compile_one(name: str) -> Path:
        obj = build_dir / (Path(name).stem + ".o")
        cmd = [compiler, *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / name), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 1)) as pool:
        objects = list(pool.map(compile_one, SOURCES))
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [compiler, *ARCH, "-shared", "-o", str(tmp), *map(str, objects)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIBRARY)
    stamp.write_text(digest)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
