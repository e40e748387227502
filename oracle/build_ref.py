"""Compile the reference's own CUDA row kernels for sm_100a into ``oracle/_ref`` (test-only).

TEST INFRASTRUCTURE ONLY.  The reference ships its row operators as two single-file
PyTorch extensions, ``src/loraforge/ops/csrc/lora_rows.cu`` (``row_shrink`` /
``row_expand``) and ``src/loraforge/ops/csrc/rowexpand.cu`` (the fleet backend's
``direct_shrink`` / ``row_expand``).  Its own build (``src/loraforge/ops/_row_extension.py``)
JIT-compiles them through ``torch.utils.cpp_extension.load``; this recipe instead calls
nvcc once per file on the sources where they lie, with the installed PyTorch's headers
and libraries and ``-gencode arch=compute_100a,code=sm_100a`` (the reference has no
Blackwell flag of its own), and writes two importable modules:

    oracle/_ref/lf_ref_rows<ext>       from lora_rows.cu   (functions shrink, expand)
    oracle/_ref/lf_ref_rowexpand<ext>  from rowexpand.cu   (functions shrink, expand)

Nothing is copied out of the reference tree and nothing is built there.  The GPU tests
use the modules as an on-device parity check and ``bench.py`` times them next to this
repository's kernels; the product never loads them.

    python oracle/build_ref.py [/path/to/loraforge]
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
MODULES = {"lf_ref_rows": "lora_rows.cu", "lf_ref_rowexpand": "rowexpand.cu"}
ARCH = ("-gencode", "arch=compute_100a,code=sm_100a")


def default_source() -> Path | None:
    """The reference tree when it is mounted (only in the build container)."""
    for candidate in (os.environ.get("LORAFORGE_REFERENCE"), "/root/reference"):
        if candidate and (Path(candidate) / "src/loraforge/ops/csrc/lora_rows.cu").exists():
            return Path(candidate)
    return None


def _command(source: Path, name: str, output: Path) -> list[str]:
    import torch
    from torch.utils import cpp_extension

    nvcc = shutil.which("nvcc") or str(Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    includes = [*cpp_extension.include_paths(device_type="cuda"), sysconfig.get_paths()["include"]]
    libs = cpp_extension.library_paths(device_type="cuda")
    cmd = [nvcc, *ARCH, "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
           f"-DTORCH_EXTENSION_NAME={name}", "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    for inc in includes:
        cmd += ["-isystem", inc]
    cmd += [str(source), "-o", str(output)]
    for lib in libs:
        cmd += ["-L", lib, "-Xlinker", f"-rpath={lib}"]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart"]
    return cmd


def build(reference: Path | None = None, force: bool = False) -> list[Path]:
    """Build both modules (skipped when their sources and this recipe are unchanged)."""
    reference = reference or default_source()
    if reference is None:
        raise FileNotFoundError("reference tree not found (set LORAFORGE_REFERENCE)")
    csrc = reference / "src/loraforge/ops/csrc"
    OUT.mkdir(exist_ok=True)
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    jobs = []
    for name, file in MODULES.items():
        source = csrc / file
        output = OUT / f"{name}{suffix}"
        stamp = OUT / f"{name}.sha256"
        digest = hashlib.sha256(source.read_bytes() + Path(__file__).read_bytes()).hexdigest()
        if not force and output.exists() and stamp.exists() and stamp.read_text() == digest:
            continue
        jobs.append((source, name, output, stamp, digest))

    def one(job):
        source, name, output, stamp, digest = job
        subprocess.run(_command(source, name, output), check=True)
        stamp.write_text(digest)
        return output

    with ThreadPoolExecutor(max_workers=2) as pool:
        list(pool.map(one, jobs))
    return [OUT / f"{name}{suffix}" for name in MODULES]


def load(name: str):
    """Import a built module from oracle/_ref (tests and bench only); None if absent."""
    import importlib

    if not any(OUT.glob(f"{name}*.so")):
        return None
    import torch  # noqa: F401  (the modules link against the loaded libtorch)

    if str(OUT) not in sys.path:
        sys.path.insert(0, str(OUT))
    return importlib.import_module(name)


if __name__ == "__main__":
    print(build(Path(sys.argv[1]) if len(sys.argv) > 1 else None, force="--force" in sys.argv))
