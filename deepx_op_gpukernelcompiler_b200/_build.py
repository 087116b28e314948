"""Build the native engine: ``csrc/dx_api.cu`` -> ``libdeepx_fused.so`` (in-tree).

The library is compiled for sm_100a only (B200) with nvcc:

    nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -std=c++17
         -Xcompiler -fPIC -shared -I<repo>/include csrc/dx_api.cu

CUDA runtime is linked statically, so the ``.so`` has no dependency on a
particular ``libcudart`` install; the driver is reached through
``cudaGetDriverEntryPoint``.  nvcc cross-compiles without a GPU present.

Run ``python -m deepx_op_gpukernelcompiler_b200._build [--force] [-v]``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_PATH = PKG_DIR / "libdeepx_fused.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    return any(src.stat().st_mtime > lib_mtime for src in _sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the engine if any source is newer than the library."""
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        _nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-shared", f"-I{INCLUDE}",
        "-o", str(tmp), str(CSRC / "dx_api.cu"),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose:
        print(proc.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
