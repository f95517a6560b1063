"""Build libfnmoe.so (sm_100a) in-tree.

    python macqwen-releases_b200/build.py [--verbose]

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` and links one shared
library next to the Python package (``flashnext_b200/libfnmoe.so``), so the
built file travels with the source tree.  Rebuilds only when a source or
header is newer than the library.  Fast-math is deliberately off: the
kernels rely on IEEE float32 rounding and denormals to match the oracle.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OUT = HERE / "flashnext_b200" / "libfnmoe.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not OUT.exists():
        return True
    built = OUT.stat().st_mtime
    deps = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > built for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the CUDA library if needed and return its path."""
    if not force and not _stale():
        return OUT
    nvcc = _nvcc()
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *FLAGS, "-I", str(INCLUDE), "-dc" if False else "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = OUT.with_suffix(".so.tmp")
    link = [nvcc, *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart"]
    subprocess.run(link, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(path)
