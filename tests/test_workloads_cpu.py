"""The seeded workloads of the metric (CPU): shapes, algorithmic work and
bytes, input order and determinism, and agreement with the golden draw of the
reference's own CPU configuration."""
import math

import torch

from deepx_op_gpukernelcompiler_b200.workloads import WORKLOADS, make_inputs
from golden_data import cases, load


def test_workload_set_and_work():
    names = set(WORKLOADS)
    assert {"linear_relu_256x512x512_f32", "linear_gelu_tanh_4096x4096x4096_bf16",
            "ffn_up_silu_8192x4096x14336_bf16", "decode_gelu_erf_16x8192x28672_f16",
            "mlp_residual_16384x4096x16384_bf16", "ffn_gated_silu_8192x4096x14336_bf16"} <= names
    w = WORKLOADS["ffn_up_silu_8192x4096x14336_bf16"]
    assert w.flops == 2 * 8192 * 4096 * 14336 == 962072674304
    d = WORKLOADS["decode_gelu_erf_16x8192x28672_f16"]
    assert d.min_bytes == 470999040  # W 469.76 MB + X + b + Y, fp16
    g = WORKLOADS["ffn_gated_silu_8192x4096x14336_bf16"]
    assert g.flops == 2 * w.flops
    assert g.min_bytes == 2 * (8192 * 4096 + 2 * 4096 * 14336 + 2 * 14336 + 8192 * 14336)
    m = WORKLOADS["mlp_residual_16384x4096x16384_bf16"]
    assert m.flops == 4 * 16384 * 4096 * 16384


def test_inputs_are_seeded_and_ordered():
    w = WORKLOADS["ffn_gated_silu_8192x4096x14336_bf16"]
    a = make_inputs(w, M=16, N=128)
    b = make_inputs(w, M=16, N=128)
    assert list(a) == ["X", "Wg", "bg", "Wu", "bu"]
    assert all(torch.equal(a[k], b[k]) for k in a)
    assert a["Wg"].dtype == torch.bfloat16 and a["Wg"].shape == (4096, 128)
    # Draw order X, Wg, bg, Wu, bu from one generator.
    g = torch.Generator().manual_seed(w.seed)
    X = torch.randn(16, 4096, generator=g)
    Wg = torch.randn(4096, 128, generator=g) / math.sqrt(4096)
    assert torch.equal(a["X"], X.bfloat16()) and torch.equal(a["Wg"], Wg.bfloat16())


def test_cpu_configuration_matches_golden_draw():
    """The reference's CPU configuration drawn by make_inputs is the golden
    fixture's input (tests/golden, from the reference's own expression)."""
    w = WORKLOADS["linear_relu_256x512x512_f32"]
    inp = make_inputs(w)
    t = load(next(c for c in cases() if c["name"] == "linear_relu_256x512x512_f32"))
    assert torch.equal(inp["X"], t["X"]) and torch.equal(inp["bias"], t["bias"])
    # W ~ N(0, 1/K): make_inputs multiplies the draw by 1/sqrt(K), the golden
    # generator divides by sqrt(K) — the same draw to within one ulp.
    assert torch.allclose(inp["W"], t["W"], rtol=2.0 ** -23, atol=0.0)
