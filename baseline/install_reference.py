"""Installs the reference package, unmodified, into ``baseline/_ref``.

    python baseline/install_reference.py <reference source dir>
    (or DEEPX_REFERENCE_DIR=<dir> python baseline/install_reference.py)

The install is pip's, offline, of a temporary copy of the source tree (the
setuptools build writes into the tree it builds), without dependencies: the
reference's own modules land in ``baseline/_ref/deepx_op_gpukernelcompiler``
and nothing of them is changed.  ``baseline/_ref`` is git-ignored; it travels
with the repository snapshot to the GPU machine, where

* ``bench.py`` times the reference's Triton and TileLang engines from it
  (``extra.reference_gpu_engines``), and
* ``tests/test_reference_harness.py`` runs the reference's own
  ``compile_and_test`` / workflow with this engine registered in its
  ``ENGINES``.

Its ``kvspace`` dependency (kvspace-py) is not in this image; the test
supplies this package's in-process KVSpace in its place.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

TARGET = Path(__file__).resolve().parent / "_ref"
PACKAGE = "deepx_op_gpukernelcompiler"


def installed() -> bool:
    return (TARGET / PACKAGE / "kernel.py").exists()


def install(src: str | os.PathLike, force: bool = False) -> Path:
    src = Path(src)
    if not (src / "pyproject.toml").exists() or not (src / PACKAGE).is_dir():
        raise FileNotFoundError(f"{src} is not the reference source tree")
    if installed() and not force:
        return TARGET
    with tempfile.TemporaryDirectory() as tmp:
        copy = Path(tmp) / "src"
        shutil.copytree(src, copy)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
               "--no-deps", "--find-links", "/opt/wheelhouse", "--upgrade",
               "--target", str(TARGET), str(copy)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"reference install failed:\n{proc.stdout}\n{proc.stderr}")
    return TARGET


if __name__ == "__main__":
    where = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DEEPX_REFERENCE_DIR")
    if not where:
        sys.exit("usage: install_reference.py <reference source dir> (or DEEPX_REFERENCE_DIR)")
    print(install(where, force="--force" in sys.argv))
