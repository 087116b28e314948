"""The oracle against the reference's own outputs (CPU).

tests/golden/ holds inputs and outputs of the reference oracle expression
(kernel.py:64-66 + fusion.py:87-92, evaluated by importing the reference;
see tests/golden/make_golden.py).  Both oracle restatements must reproduce
them before they are trusted as the checker of the GPU kernels.
"""
import numpy as np
import pytest
import torch

import oracle
from golden_data import cases, load

# The golden outputs were evaluated in fp32 by torch; the oracle differs only
# by fp32 summation order (f32 path) or by being exact (f64 path).
ORACLE_RTOL = 2e-5
ORACLE_ATOL = 2e-5


def _run(case, fn):
    t = load(case)
    if case["mlp"]:
        return fn["mlp"](t["X"], t["W1"], t["b1"], t["W2"], t["b2"], case["act"]), t["Y"]
    if case.get("gated"):
        if case["ffn"]:
            return fn["ffn_gated"](t["X"], t["Wg"], t["bg"], t["Wu"], t["bu"], t["Wo"], t["bo"],
                                   case["act"]), t["Y"]
        return fn["gated"](t["X"], t["Wg"], t["bg"], t["Wu"], t["bu"], case["act"]), t["Y"]
    return fn["linear"](t["X"], t["W"], t["bias"], case["act"], residual=t.get("R")), t["Y"]


F64 = {"linear": oracle.fused_linear_f64, "mlp": oracle.mlp_residual_f64,
       "gated": oracle.gated_linear_f64, "ffn_gated": oracle.gated_ffn_f64}
F32 = {"linear": oracle.fused_linear_f32, "mlp": oracle.mlp_residual_f32,
       "gated": oracle.gated_linear_f32, "ffn_gated": oracle.gated_ffn_f32}


def _torch_linear(X, W, b, act, residual=None):
    return oracle.torch_cpu.fused_linear(X, W, b, act, residual=residual).numpy()


@pytest.mark.parametrize("case", [c for c in cases() if not c.get("gated")],
                         ids=lambda c: c["name"])
def test_oracle_torch_cpu_matches_reference(case):
    """The torch-CPU restatement timed as the CPU baseline."""
    fn = {"linear": _torch_linear,
          "mlp": lambda *a: oracle.torch_cpu.mlp_residual(*a).numpy()}
    got, ref = _run(case, fn)
    np.testing.assert_allclose(got, ref.numpy(), rtol=ORACLE_RTOL, atol=ORACLE_ATOL)


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_oracle_f64_matches_reference(case):
    got, ref = _run(case, F64)
    np.testing.assert_allclose(got, ref.numpy(), rtol=ORACLE_RTOL, atol=ORACLE_ATOL)


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_oracle_f32_matches_reference(case):
    got, ref = _run(case, F32)
    np.testing.assert_allclose(got, ref.numpy(), rtol=ORACLE_RTOL, atol=ORACLE_ATOL)


def test_golden_covers_every_compilable_activation():
    acts = {c["act"] for c in cases()}
    assert {None, "relu", "gelu", "silu", "swish", "gelu_erf"} <= acts
    assert {c["dtype"] for c in cases()} == {"f32", "f16", "bf16"}
    assert any(c["residual"] for c in cases()) and any(c["mlp"] for c in cases())
    assert any(c.get("gated") and c["ffn"] for c in cases())


def test_reference_cpu_config_is_pinned():
    """ReLU(X[256,512] W[512,512] + b), fp32, seed 0: inputs are the seeded draw."""
    case = next(c for c in cases() if c["name"] == "linear_relu_256x512x512_f32")
    t = load(case)
    g = torch.Generator().manual_seed(0)
    X = torch.randn(256, 512, generator=g)
    W = torch.randn(512, 512, generator=g) / 512 ** 0.5
    b = torch.rand(512, generator=g) * 0.2 - 0.1
    assert torch.equal(t["X"], X) and torch.equal(t["W"], W) and torch.equal(t["bias"], b)


def test_planted_activation_mistake_is_caught():
    """Swap tanh-GELU for erf-GELU inside the oracle: the golden check must fail."""
    case = next(c for c in cases() if c["act"] == "gelu" and c["dtype"] == "f32")
    t = load(case)
    wrong = oracle.fused_linear_f64(t["X"], t["W"], t["bias"], "gelu_erf")
    err = np.abs(wrong - t["Y"].numpy()).max()
    assert err > 10 * ORACLE_ATOL


def test_planted_gate_mistake_is_caught():
    """Apply the activation to the up projection instead of the gate."""
    case = next(c for c in cases() if c.get("gated") and c["dtype"] == "f32")
    t = load(case)
    wrong = (oracle.fused_linear_f64(t["X"], t["Wg"], t["bg"], None)
             * oracle.fused_linear_f64(t["X"], t["Wu"], t["bu"], case["act"]))
    assert np.abs(wrong - t["Y"].numpy()).max() > 10 * ORACLE_ATOL


def test_planted_bias_mistake_is_caught():
    case = next(c for c in cases() if c["act"] == "relu" and c["dtype"] == "f32")
    t = load(case)
    wrong = oracle.fused_linear_f64(t["X"], t["W"], None, "relu")
    assert np.abs(wrong - t["Y"].numpy()).max() > 10 * ORACLE_ATOL


def test_activation_formulas():
    x = np.linspace(-8, 8, 1001)
    t = torch.from_numpy(x)
    np.testing.assert_allclose(oracle.activation_f64(x, "relu"), np.maximum(x, 0))
    np.testing.assert_allclose(oracle.activation_f64(x, "gelu"),
                               torch.nn.functional.gelu(t, approximate="tanh").numpy(), atol=1e-12)
    np.testing.assert_allclose(oracle.activation_f64(x, "gelu_erf"),
                               torch.nn.functional.gelu(t).numpy(), atol=1e-12)
    np.testing.assert_allclose(oracle.activation_f64(x, "silu"),
                               torch.nn.functional.silu(t).numpy(), atol=1e-12)


def test_oracle_edge_shapes():
    assert oracle.fused_linear_f64(np.zeros((0, 4)), np.zeros((4, 3)), None).shape == (0, 3)
    y = oracle.fused_linear_f64(np.zeros((2, 0)), np.zeros((0, 3)), np.array([1.0, -2.0, 3.0]), "relu")
    np.testing.assert_array_equal(y, [[1, 0, 3], [1, 0, 3]])
    with pytest.raises(ValueError):
        oracle.fused_linear_f64(np.zeros((2, 3)), np.zeros((4, 3)))
