"""Builds the sm_100a shared library of the paged-attention path in-tree.

    python -m batchstream_inference_engine_b200.build

compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` only and links
``libbatchstream_b200.so`` next to this file.  The CUDA runtime is linked
statically and its symbols are kept local to the library, so the library does
not depend on (or interfere with) the runtime that PyTorch loads; the driver is
reached at run time through the runtime's entry-point query, so the library
also loads on a machine without a GPU driver.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
BUILD = PACKAGE / "_build"
LIBRARY = PACKAGE / "libbatchstream_b200.so"
INCLUDE = PACKAGE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build the library")
    return found


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(src.stat().st_mtime > mtime for src in sources)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile (if stale) and return the path of the shared library."""
    BUILD.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    sources = sorted(CSRC.glob("*.cu"))
    compiler = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if force or _stale(obj, [src, *headers]):
            cmd = [compiler, *ARCH, *CFLAGS, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            proc = subprocess.run(cmd, capture_output=True, text=True)
            if proc.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stderr}")
            if verbose and proc.stderr:
                print(proc.stderr, file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(compile_one, sources))

    if force or _stale(LIBRARY, objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [
            compiler, *ARCH, "-shared", "-cudart", "static",
            "-Xlinker", "--exclude-libs,ALL", "-Xlinker", "-Bsymbolic",
            *[str(o) for o in objects], "-o", str(tmp),
        ]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"linking libbatchstream_b200.so failed:\n{proc.stderr}")
        tmp.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="--force" in sys.argv))
