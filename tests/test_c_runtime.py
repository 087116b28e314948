"""The engine from a non-Python caller: tests/c_runtime/dx_runtime_demo.cpp
dlopens libdeepx_fused.so, compiles plans and calls them with raw device
pointers (the design docs' C++ runtime, doc/kernel-compiler-analysis.md:113-134).
Building it needs only g++ and the CUDA headers (CPU); running it needs a GPU."""
import shutil
import subprocess
from pathlib import Path

import pytest
import torch

from deepx_op_gpukernelcompiler_b200 import _build, _native as nat

ROOT = Path(__file__).resolve().parent.parent
SRC = Path(__file__).resolve().parent / "c_runtime" / "dx_runtime_demo.cpp"
CUDA = Path("/usr/local/cuda")


def _compile(out: Path) -> Path:
    gxx = shutil.which("g++")
    if gxx is None or not (CUDA / "include" / "cuda_runtime.h").exists():
        pytest.skip("g++ or the CUDA toolkit headers are missing")
    lib_dirs = [d for d in (CUDA / "lib64", CUDA / "targets" / "x86_64-linux" / "lib") if d.exists()]
    cmd = [gxx, "-O2", "-std=c++17", str(SRC), f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}",
           *(f"-L{d}" for d in lib_dirs), *(f"-Wl,-rpath,{d}" for d in lib_dirs),
           "-lcudart", "-ldl", "-o", str(out)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr[-3000:]
    return out


def test_runtime_demo_builds(tmp_path):
    assert _compile(tmp_path / "dx_runtime_demo").exists()


@pytest.mark.gpu
def test_runtime_demo_runs_plans(tmp_path):
    assert torch.cuda.is_available()
    _build.build()
    exe = _compile(tmp_path / "dx_runtime_demo")
    proc = subprocess.run([str(exe), str(nat.LIB_PATH)], capture_output=True, text=True,
                          timeout=300)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    lines = proc.stdout.splitlines()
    assert lines[0] == "engine ABI version 100"
    assert any(l.startswith("linear_relu M=512") and "bad=0" in l for l in lines)
    assert any(l.startswith("linear_gelu M=16") and "bad=0" in l and "workspace=0" not in l
               for l in lines)
    assert any(l.startswith("mlp_residual M=256") and "bad=0" in l for l in lines)
