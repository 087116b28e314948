"""ORACLE — test infrastructure only (bench.py's CPU baseline and reference
arm, and tests).  Nothing in the engine imports this module.

The reference's own CPU expression, restated in torch on the host cores:

    ref = a @ b + bias                      (kernel.py:64)
    ref = ACTIVATION_PT[activation](ref)    (kernel.py:65-66)

with ACTIVATION_PT as fusion.py:87-92 defines it — relu; gelu with the tanh
approximation; silu; swish = silu — plus gelu_erf (F.gelu without
approximation, the form kernel_triton.py:61 computes) for the decode
configuration, and the residual add of the MLP chain.  The arithmetic is
torch's fp32 CPU matmul (the library the reference's oracle runs on),
threaded over `threads` host cores.
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

ACTIVATIONS = {
    None: lambda t: t,
    "none": lambda t: t,
    "relu": torch.relu,
    "gelu": lambda t: F.gelu(t, approximate="tanh"),
    "gelu_tanh": lambda t: F.gelu(t, approximate="tanh"),
    "gelu_erf": F.gelu,
    "silu": F.silu,
    "swish": F.silu,
}


def host_threads() -> int:
    """Host cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def use_threads(n: int | None = None) -> int:
    """Set torch's intra-op thread count (torchrun sets OMP_NUM_THREADS=1 for
    its ranks, which would leave the baseline on one core) and return it."""
    torch.set_num_threads(max(1, n or host_threads()))
    return torch.get_num_threads()


def fused_linear(X: torch.Tensor, W: torch.Tensor, bias: torch.Tensor | None,
                 activation=None, residual: torch.Tensor | None = None) -> torch.Tensor:
    """act(X @ W + bias) (+ residual) in fp32 on the CPU."""
    ref = X.float() @ W.float()
    if bias is not None:
        ref = ref + bias.float()
    ref = ACTIVATIONS[activation](ref)
    if residual is not None:
        ref = ref + residual.float()
    return ref


def mlp_residual(X, W1, b1, W2, b2, activation="gelu") -> torch.Tensor:
    """Y = act(X W1 + b1) W2 + b2 + X in fp32 on the CPU."""
    H = fused_linear(X, W1, b1, activation)
    return fused_linear(H, W2, b2, None, residual=X)
