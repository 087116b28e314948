"""Two-GEMM FFN chains, each GEMM one fused launch.

``mlp_residual`` — the chain matmul -> add -> gelu -> matmul -> add -> add:

    H = act(X @ W1 + b1)          fused launch 1 (bias + activation epilogue)
    Y = H @ W2 + b2 + X           fused launch 2 (bias + residual epilogue)

This is the opcode chain matmul -> add -> gelu -> matmul -> add -> add.  The
reference classifies its nearest relative, ``ffn_two_layer``, as
multi_kernel and does not run it (deepx_op_gpukernelcompiler/kernel.py:45-46);
here each GEMM is one fused kernel and the intermediate H makes one HBM round
trip.  GELU is the tanh form, as ``ACTIVATION_PT['gelu']`` (fusion.py:89).

``gated_ffn`` — the ``ffn_gated`` chain (fusion.py:44-46; fixtures
test/fusion_cases/07_ffn_gated.kv, 08_ffn_swiglu.kv):

    H = silu(X @ Wg + bg) * (X @ Wu + bu)   one dual-GEMM launch
    Y = H @ Wo + bo                         one fused linear launch

``two_layer_ffn`` — the ``ffn_two_layer`` chain (fusion.py:42-43):
Y = relu(X @ W1 + b1) @ W2 + b2, two fused launches.
"""
from __future__ import annotations

import torch

from .linear import fused_gated_linear, fused_linear


def mlp_residual(X: torch.Tensor, W1: torch.Tensor, b1: torch.Tensor | None,
                 W2: torch.Tensor, b2: torch.Tensor | None, activation="gelu",
                 hidden: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Y = act(X W1 + b1) W2 + b2 + X.  `hidden` optionally receives H."""
    if W2.shape[1] != X.shape[1]:
        raise ValueError(f"W2 must map back to X's width {X.shape[1]}, got {tuple(W2.shape)}")
    H = fused_linear(X, W1, b1, activation, out=hidden)
    return fused_linear(H, W2, b2, None, residual=X, out=out)


def gated_ffn(X: torch.Tensor, Wg: torch.Tensor, bg: torch.Tensor | None, Wu: torch.Tensor,
              bu: torch.Tensor | None, Wo: torch.Tensor, bo: torch.Tensor | None,
              activation="silu", hidden: torch.Tensor | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Y = (act(X Wg + bg) * (X Wu + bu)) Wo + bo.  `hidden` optionally receives H."""
    if Wo.shape[0] != Wg.shape[1]:
        raise ValueError(f"Wo must take the hidden width {Wg.shape[1]}, got {tuple(Wo.shape)}")
    H = fused_gated_linear(X, Wg, Wu, bg, bu, activation, out=hidden)
    return fused_linear(H, Wo, bo, None, out=out)


def two_layer_ffn(X: torch.Tensor, W1: torch.Tensor, b1: torch.Tensor | None, W2: torch.Tensor,
                  b2: torch.Tensor | None, activation="relu",
                  hidden: torch.Tensor | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Y = act(X W1 + b1) W2 + b2 (no residual)."""
    H = fused_linear(X, W1, b1, activation, out=hidden)
    return fused_linear(H, W2, b2, None, out=out)
