"""ORACLE build recipe (test infrastructure only).

Compiles ``oracle/fused_linear_ref.c`` with gcc into
``oracle/liboracle_fused.so`` (git-ignored; it travels with the repo
snapshot like the engine library):

    gcc -O2 -fopenmp -fPIC -shared -o oracle/liboracle_fused.so \
        oracle/fused_linear_ref.c -lm

The reference itself is Python (no C/C++ path to compile), so there is no
``oracle/_ref`` build; golden vectors come from importing the reference's
Python in ``tests/golden/make_golden.py``.
"""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
SRC = ORACLE_DIR / "fused_linear_ref.c"
LIB = ORACLE_DIR / "liboracle_fused.so"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("gcc not found")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, "-O2", "-fopenmp", "-fPIC", "-shared", "-o", str(tmp), str(SRC), "-lm"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{proc.stdout}\n{proc.stderr}")
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
