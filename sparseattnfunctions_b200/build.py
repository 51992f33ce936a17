"""Builds the CUDA library ``libsaf.so`` in-tree for sm_100a.

Every ``csrc/*.cu`` file is compiled with nvcc to an object under ``_build/``
at the repository root and linked into ``sparseattnfunctions_b200/libsaf.so``.
The library links the CUDA runtime statically and reaches the driver API only
through ``cudaGetDriverEntryPoint``, so it needs no libcuda at link time and
cross-compiles on a machine without a GPU.

    python -m sparseattnfunctions_b200.build
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = REPO_DIR / "_build"
LIB_PATH = PKG_DIR / "libsaf.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _compile(nvcc: str, src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr)
    return obj


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compiles every ``csrc/*.cu`` and links ``libsaf.so``; returns its path.

    Skips the work when the library is newer than every source and header,
    unless ``force`` is set.
    """
    sources = sorted(CSRC.glob("*.cu"))
    deps = sources + sorted(CSRC.glob("*.cuh")) + sorted((REPO_DIR / "include").glob("*.h"))
    if (not force and LIB_PATH.exists()
            and all(LIB_PATH.stat().st_mtime >= d.stat().st_mtime for d in deps)):
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    nvcc = nvcc_path()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, verbose), sources))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(path)
