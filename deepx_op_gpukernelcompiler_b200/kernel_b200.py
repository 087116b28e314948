"""B200 engine factory, the drop-in for the reference's kernel generators.

``make_linear_kernel(activation)`` has the reference's factory shape
(kernel_triton.py:70-89): it returns ``kernel_fn(A, B, bias) -> C`` with
C = act(A @ B + bias), A[M,K], B[K,N], bias[N], C allocated with A's dtype.
There is no JIT or autotune step — the sm_100a kernels are prebuilt and pick
their tiling from the shape — so the TileLang form
``kernel_fn(M, N, K, BM, BN, BK, dtype, accum)`` (kernel_tilelang.py:26-27)
is not needed.  ``kernel_fn`` additionally accepts ``residual=`` (added after
the activation) and ``out=`` (a preallocated C).
"""
from __future__ import annotations

import torch

from .linear import activation_code, fused_linear


def make_linear_kernel(activation: str | None = None):
    """Return ``kernel_fn(A, B, bias=None, residual=None, out=None) -> C``."""
    activation_code(activation)  # reject unknown names at factory time

    def kernel_fn(A: torch.Tensor, B: torch.Tensor, bias: torch.Tensor | None = None,
                  residual: torch.Tensor | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
        return fused_linear(A, B, bias, activation, residual=residual, out=out)

    kernel_fn.activation = activation
    return kernel_fn
