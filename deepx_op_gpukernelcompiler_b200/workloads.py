"""Seeded synthetic workloads of the fused-linear hot path.

Each workload is a fused linear (or the two-layer MLP chain, or the gated
dual GEMM) at a fixed shape, dtype, activation and seed.  Inputs are drawn
with a torch Generator seeded with the workload's seed, in the order X, W,
bias (MLP: X, W1, b1, W2, b2; gated: X, Wg, bg, Wu, bu): X ~ N(0, 1),
W ~ N(0, 1/fan_in), bias ~ U(-0.1, 0.1), generated in fp32 and then cast to
the workload dtype.  Comparisons use the cast inputs
upcast back to fp32.

Tolerances: fp32 rtol = atol = 1e-4; fp16/bf16 (fp32 accumulate) rtol =
atol = 2e-2, both against an fp32 evaluation of the same expression.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
TOLERANCE = {"f32": (1e-4, 1e-4), "f16": (2e-2, 2e-2), "bf16": (2e-2, 2e-2)}


@dataclass(frozen=True)
class Workload:
    name: str
    M: int
    K: int
    N: int
    dtype: str
    act: str | None
    seed: int
    mlp: bool = False  # two-layer chain: Y = act(X W1 + b1) W2 + b2 + X
    gated: bool = False  # dual GEMM: Y = act(X Wg + bg) * (X Wu + bu)

    @property
    def torch_dtype(self) -> torch.dtype:
        return DTYPES[self.dtype]

    @property
    def flops(self) -> int:
        """Algorithmic GEMM work, 2*M*N*K per GEMM (epilogue excluded)."""
        return (4 if (self.mlp or self.gated) else 2) * self.M * self.N * self.K

    @property
    def min_bytes(self) -> int:
        """Bytes that must cross HBM once: inputs read + output written."""
        e = torch.finfo(self.torch_dtype).bits // 8
        if self.mlp:
            return e * (2 * self.M * self.K + 2 * self.K * self.N + self.N + self.K
                        + self.M * self.K)
        if self.gated:
            return e * (self.M * self.K + 2 * self.K * self.N + 2 * self.N + self.M * self.N)
        return e * (self.M * self.K + self.K * self.N + self.N + self.M * self.N)

    @property
    def tolerance(self) -> tuple[float, float]:
        return TOLERANCE[self.dtype]


WORKLOADS = {
    w.name: w for w in [
        Workload("linear_relu_256x512x512_f32", 256, 512, 512, "f32", "relu", 0),
        Workload("linear_gelu_tanh_4096x4096x4096_bf16", 4096, 4096, 4096, "bf16", "gelu_tanh", 1),
        Workload("ffn_up_silu_8192x4096x14336_bf16", 8192, 4096, 14336, "bf16", "silu", 2),
        Workload("decode_gelu_erf_16x8192x28672_f16", 16, 8192, 28672, "f16", "gelu_erf", 3),
        Workload("mlp_residual_16384x4096x16384_bf16", 16384, 4096, 16384, "bf16", "gelu_tanh", 4,
                 mlp=True),
        Workload("ffn_gated_silu_8192x4096x14336_bf16", 8192, 4096, 14336, "bf16", "silu", 5,
                 gated=True),
    ]
}


def make_inputs(w: Workload, device="cpu", M: int | None = None,
                N: int | None = None) -> dict[str, torch.Tensor]:
    """Seeded inputs in the workload dtype.  `M`/`N` override the sizes
    (same distributions) for scaled-down parity cases."""
    M = w.M if M is None else M
    N = w.N if N is None else N
    K = w.K
    gen = torch.Generator(device=device)
    gen.manual_seed(w.seed)
    dt = w.torch_dtype

    def normal(*shape, std=1.0):
        return (torch.randn(shape, generator=gen, device=device) * std).to(dt)

    def uniform(*shape):
        return (torch.rand(shape, generator=gen, device=device) * 0.2 - 0.1).to(dt)

    if w.mlp:
        X = normal(M, K)
        W1 = normal(K, N, std=1.0 / math.sqrt(K))
        b1 = uniform(N)
        W2 = normal(N, K, std=1.0 / math.sqrt(N))
        b2 = uniform(K)
        return {"X": X, "W1": W1, "b1": b1, "W2": W2, "b2": b2}
    X = normal(M, K)
    W = normal(K, N, std=1.0 / math.sqrt(K))
    b = uniform(N)
    if w.gated:
        Wu = normal(K, N, std=1.0 / math.sqrt(K))
        bu = uniform(N)
        return {"X": X, "Wg": W, "bg": b, "Wu": Wu, "bu": bu}
    return {"X": X, "W": W, "bias": b}
