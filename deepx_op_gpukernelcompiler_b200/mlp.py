"""Two-layer MLP chain with residual: the ``mlp_residual`` fusion pattern.

    H = act(X @ W1 + b1)          fused launch 1 (bias + activation epilogue)
    Y = H @ W2 + b2 + X           fused launch 2 (bias + residual epilogue)

This is the opcode chain matmul -> add -> gelu -> matmul -> add -> add.  The
reference classifies its nearest relative, ``ffn_two_layer``, as
multi_kernel and does not run it (deepx_op_gpukernelcompiler/kernel.py:45-46);
here each GEMM is one fused kernel and the intermediate H makes one HBM round
trip.  GELU is the tanh form, as ``ACTIVATION_PT['gelu']`` (fusion.py:89).
"""
from __future__ import annotations

import torch

from .linear import fused_linear


def mlp_residual(X: torch.Tensor, W1: torch.Tensor, b1: torch.Tensor | None,
                 W2: torch.Tensor, b2: torch.Tensor | None, activation="gelu",
                 hidden: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Y = act(X W1 + b1) W2 + b2 + X.  `hidden` optionally receives H."""
    if W2.shape[1] != X.shape[1]:
        raise ValueError(f"W2 must map back to X's width {X.shape[1]}, got {tuple(W2.shape)}")
    H = fused_linear(X, W1, b1, activation, out=hidden)
    return fused_linear(H, W2, b2, None, residual=X, out=out)
