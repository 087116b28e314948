"""Parity at the workloads' full sizes (gpu).

Every configuration of the metric at its own size and seed
(workloads.WORKLOADS: inputs drawn in the order X, W, bias on a seeded CPU
generator, fp32 then cast): the engine's output against the reference
expression act(a @ b + bias) (kernel.py:64-66, fusion.py:87-92) evaluated in
fp32 on the GPU with TF32 off over the whole output, and against the fp64 C
oracle on random row blocks.  Tolerances: fp32 rtol = atol = 1e-4; fp16/bf16
rtol = atol = 2e-2.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from deepx_op_gpukernelcompiler_b200 import _native as nat
from deepx_op_gpukernelcompiler_b200 import fused_gated_linear, fused_linear, mlp_residual
from deepx_op_gpukernelcompiler_b200.workloads import WORKLOADS, make_inputs

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")

ACT_FP32 = {
    None: lambda v: v,
    "relu": torch.relu,
    "gelu_tanh": lambda v: F.gelu(v, approximate="tanh"),
    "gelu_erf": lambda v: F.gelu(v),
    "silu": F.silu,
}


def _fp32_linear(X, W, b, act, R=None):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        Y = ACT_FP32[act](X.float() @ W.float() + b.float())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return Y + R.float() if R is not None else Y


def _check(got, ref, tol, what):
    rtol, atol = tol
    err = (got.float() - ref).abs()
    bad = err > atol + rtol * ref.abs()
    assert not bool(bad.any()), (f"{what}: {int(bad.sum())} of {bad.numel()} elements off; max "
                                 f"|diff| {err.max().item():.4g}")


@pytest.mark.parametrize("name", [n for n, w in WORKLOADS.items() if not (w.mlp or w.gated)])
def test_fullsize_linear(name):
    w = WORKLOADS[name]
    inp = make_inputs(w)  # CPU, seeded
    X, W, b = (inp[k].to(DEV) for k in ("X", "W", "bias"))
    Y = fused_linear(X, W, b, w.act)
    plan = nat.last_launch_plan()
    ref = _fp32_linear(X, W, b, w.act)
    torch.cuda.synchronize()
    _check(Y, ref, w.tolerance, f"{name} [{plan.split()[0]}] vs fp32 expression")
    # fp64 C oracle on three random row blocks of 8 rows.
    rng = np.random.default_rng(w.seed)
    for r0 in sorted(set(int(v) for v in rng.integers(0, max(1, w.M - 8), size=3))):
        r1 = min(w.M, r0 + 8)
        ref64 = oracle.fused_linear_f64(inp["X"][r0:r1], inp["W"], inp["bias"], w.act)
        _check(Y[r0:r1].cpu(), torch.from_numpy(ref64).float(), w.tolerance,
               f"{name} rows {r0}:{r1} vs fp64 oracle")


def test_fullsize_mlp_chain():
    w = next(w for w in WORKLOADS.values() if w.mlp)
    inp = make_inputs(w)
    X, W1, b1, W2, b2 = (inp[k].to(DEV) for k in ("X", "W1", "b1", "W2", "b2"))
    Y = mlp_residual(X, W1, b1, W2, b2, w.act)
    # fp32 chain from the same rounded inputs; the engine rounds H to bf16
    # between the two launches, as the reference's two separate ops would.
    H = _fp32_linear(X, W1, b1, w.act).to(X.dtype)
    ref = _fp32_linear(H, W2, b2, None, R=X)
    torch.cuda.synchronize()
    _check(Y, ref, w.tolerance, f"{w.name} vs fp32 chain")


def test_fullsize_gated():
    w = next(w for w in WORKLOADS.values() if w.gated)
    inp = make_inputs(w)
    X, Wg, bg, Wu, bu = (inp[k].to(DEV) for k in ("X", "Wg", "bg", "Wu", "bu"))
    Y = fused_gated_linear(X, Wg, Wu, bg, bu, w.act)
    plan = nat.last_launch_plan()
    ref = _fp32_linear(X, Wg, bg, w.act) * _fp32_linear(X, Wu, bu, None)
    torch.cuda.synchronize()
    _check(Y, ref, w.tolerance, f"{w.name} [{plan.split()[0]}] vs fp32 expression")
    r0 = int(np.random.default_rng(w.seed).integers(0, w.M - 8))
    ref64 = oracle.gated_linear_f64(inp["X"][r0:r0 + 8], inp["Wg"], inp["bg"], inp["Wu"],
                                    inp["bu"], w.act)
    _check(Y[r0:r0 + 8].cpu(), torch.from_numpy(ref64).float(), w.tolerance,
           f"{w.name} rows {r0}:{r0 + 8} vs fp64 oracle")
