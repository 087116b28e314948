"""Gated dual GEMM and the ffn_gated chain on the GPU, through the C ABI (gpu).

Y = act(X Wg + bg) * (X Wu + bu) (dx_fused_gated_linear) against the golden
outputs generated from the reference's own activation table and against the
fp64 oracle, for every kernel variant, at the workloads' tolerances: fp32
rtol = atol = 1e-4, fp16/bf16 rtol = atol = 2e-2.
"""
import numpy as np
import pytest
import torch

import oracle
from deepx_op_gpukernelcompiler_b200 import _native as nat
from deepx_op_gpukernelcompiler_b200 import fused_gated_linear, gated_ffn, two_layer_ffn
from golden_data import cases, load

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-4, 1e-4), torch.float16: (2e-2, 2e-2), torch.bfloat16: (2e-2, 2e-2)}
DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
DEV = torch.device("cuda:0")
# Variant forced -> the kernel name the launch plan must report.
PLAN_NAME = {"simt": "simt_gated", "umma_1cta": "umma_1cta_gated", "decode": "decode_gated"}


def _assert_close(got, ref, dtype, what=""):
    rtol, atol = TOL[dtype]
    g = got.float().cpu().numpy()
    r = ref.numpy() if isinstance(ref, torch.Tensor) else np.asarray(ref)
    bad = ~np.isclose(g, r, rtol=rtol, atol=atol)
    if bad.any():
        idx = tuple(np.argwhere(bad)[0])
        raise AssertionError(f"{what}: {bad.sum()} of {bad.size} off; first at {idx}: got {g[idx]}, "
                             f"want {r[idx]}; max |diff| {np.abs(g - r).max():.4g}")


def _variants(M, dtype):
    if dtype == torch.float32:
        return ["auto", "simt"]
    out = ["auto", "simt", "umma", "umma_1cta"]
    if M <= 64:
        out.append("decode")
    return out


def _check_plan(kern, M):
    plan = nat.last_launch_plan()
    if kern in PLAN_NAME:
        assert plan.startswith(PLAN_NAME[kern]), plan
    elif kern == "umma":
        assert plan.startswith("umma_pair_gated" if M >= 256 else "umma_1cta_gated"), plan


@pytest.mark.parametrize("case", [c for c in cases() if c.get("gated") and not c["ffn"]],
                         ids=lambda c: c["name"])
def test_golden_gated(case):
    t = {k: v.to(DEV) for k, v in load(case).items()}
    dt = DT[case["dtype"]]
    for kern in _variants(case["M"], dt):
        Y = fused_gated_linear(t["X"], t["Wg"], t["Wu"], t["bg"], t["bu"], case["act"], kernel=kern)
        torch.cuda.synchronize()
        _check_plan(kern, case["M"])
        _assert_close(Y, t["Y"].cpu(), dt, f"{case['name']} [{kern}]")
    assert nat.device_status(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize("case", [c for c in cases() if c.get("gated") and c["ffn"]],
                         ids=lambda c: c["name"])
def test_golden_ffn_gated(case):
    t = {k: v.to(DEV) for k, v in load(case).items()}
    Y = gated_ffn(t["X"], t["Wg"], t["bg"], t["Wu"], t["bu"], t["Wo"], t["bo"], case["act"])
    torch.cuda.synchronize()
    _assert_close(Y, t["Y"].cpu(), DT[case["dtype"]], case["name"])


def _rand(M, K, N, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(M, K, generator=g).to(dtype)
    Wg = (torch.randn(K, N, generator=g) / K ** 0.5).to(dtype)
    Wu = (torch.randn(K, N, generator=g) / K ** 0.5).to(dtype)
    bg = (torch.rand(N, generator=g) * 0.2 - 0.1).to(dtype)
    bu = (torch.rand(N, generator=g) * 0.2 - 0.1).to(dtype)
    return X, Wg, bg, Wu, bu


GATED_SHAPES = [  # (M, K, N): decode / single-CTA / pair regimes, ragged N and M
    (1, 64, 128), (16, 4096, 1536), (48, 520, 200), (64, 256, 3000), (65, 512, 264),
    (128, 256, 384), (255, 192, 136), (256, 1024, 1024), (300, 1000, 8), (513, 256, 760),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K,N", GATED_SHAPES)
def test_gated_shapes_all_variants(M, K, N, dtype):
    X, Wg, bg, Wu, bu = _rand(M, K, N, dtype, seed=M * 7 + N)
    ref = oracle.gated_linear_f64(X, Wg, bg, Wu, bu, "silu")
    d = [t.to(DEV) for t in (X, Wg, bg, Wu, bu)]
    for kern in _variants(M, dtype):
        Y = fused_gated_linear(d[0], d[1], d[3], d[2], d[4], "silu", kernel=kern)
        torch.cuda.synchronize()
        _check_plan(kern, M)
        _assert_close(Y, ref, dtype, f"{M}x{K}x{N} {dtype} [{kern}]")



@pytest.mark.parametrize("M,N,halves", [(16, 14336, 2), (3, 14336, 2), (16, 28672, 4), (8, 3584, 4)])
def test_gated_decode_unit_width(M, N, halves):
    """Gated M <= 16 streams 256 columns of each weight per work unit (4 UMMA
    halves), except when 128-column units give one whole tile per CTA and
    256-column units do not (N = 14336 on 148 SMs: 112 whole tiles against 56
    split ones); both widths match the oracle."""
    K = 512
    X, Wg, bg, Wu, bu = _rand(M, K, N, torch.float16, seed=M + N)
    ref = oracle.gated_linear_f64(X, Wg, bg, Wu, bu, "silu")
    d = [t.to(DEV) for t in (X, Wg, bg, Wu, bu)]
    Y = fused_gated_linear(d[0], d[1], d[3], d[2], d[4], "silu", kernel="decode")
    torch.cuda.synchronize()
    plan = nat.last_launch_plan()
    assert plan.startswith("decode_gated"), plan
    if torch.cuda.get_device_properties(DEV).multi_processor_count == 148:
        assert f"halves={halves} " in plan, plan
    _assert_close(Y, ref, torch.float16, f"{M}x{K}x{N} gated decode")

@pytest.mark.parametrize("act", ["gelu", "relu", None])
def test_gated_other_activations_no_bias(act):
    M, K, N = 200, 384, 520
    X, Wg, _, Wu, _ = _rand(M, K, N, torch.bfloat16, seed=5)
    ref = oracle.gated_linear_f64(X, Wg, None, Wu, None, act)
    for kern in ("umma", "simt"):
        Y = fused_gated_linear(X.to(DEV), Wg.to(DEV), Wu.to(DEV), None, None, act, kernel=kern)
        torch.cuda.synchronize()
        _assert_close(Y, ref, torch.bfloat16, f"{act} [{kern}]")


def test_gated_fp32_exact():
    X, Wg, bg, Wu, bu = _rand(70, 96, 130, torch.float32, seed=9)
    ref = oracle.gated_linear_f64(X, Wg, bg, Wu, bu, "silu")
    Y = fused_gated_linear(X.to(DEV), Wg.to(DEV), Wu.to(DEV), bg.to(DEV), bu.to(DEV), "silu")
    _assert_close(Y, ref, torch.float32, "fp32")


@pytest.mark.parametrize("kern,M", [("decode", 16), ("umma", 512), ("umma_1cta", 128)])
def test_gated_bitwise_deterministic(kern, M):
    X, Wg, bg, Wu, bu = (t.to(DEV) for t in _rand(M, 2048, 1024, torch.bfloat16, seed=3))
    a = fused_gated_linear(X, Wg, Wu, bg, bu, "silu", kernel=kern)
    b = fused_gated_linear(X, Wg, Wu, bg, bu, "silu", kernel=kern)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_gated_matches_two_plain_launches():
    """The dual-GEMM launch equals silu(linear) * linear built from two plain launches
    (within rounding of the materialised intermediates)."""
    from deepx_op_gpukernelcompiler_b200 import fused_linear
    X, Wg, bg, Wu, bu = (t.to(DEV) for t in _rand(384, 1024, 768, torch.bfloat16, seed=11))
    Y = fused_gated_linear(X, Wg, Wu, bg, bu, "silu")
    G = fused_linear(X, Wg, bg, "silu").float()
    U = fused_linear(X, Wu, bu, None).float()
    torch.cuda.synchronize()
    assert torch.allclose(Y.float(), G * U, rtol=2e-2, atol=2e-2)


def test_gated_decode_workspace_reuse_across_kinds():
    """Gated and plain decode launches share the per-stream workspace; tickets
    left at zero by one must serve the next."""
    from deepx_op_gpukernelcompiler_b200 import fused_linear
    X, Wg, bg, Wu, bu = _rand(16, 1024, 2048, torch.float16, seed=13)
    ref_g = oracle.gated_linear_f64(X, Wg, bg, Wu, bu, "silu")
    ref_l = oracle.fused_linear_f64(X, Wg, bg, "silu")
    d = [t.to(DEV) for t in (X, Wg, bg, Wu, bu)]
    for _ in range(2):
        Yg = fused_gated_linear(d[0], d[1], d[3], d[2], d[4], "silu", kernel="decode")
        Yl = fused_linear(d[0], d[1], d[2], "silu", kernel="decode")
        torch.cuda.synchronize()
        _assert_close(Yg, ref_g, torch.float16, "gated")
        _assert_close(Yl, ref_l, torch.float16, "plain")


def test_gated_rejects_bad_arguments():
    X, Wg, bg, Wu, bu = (t.to(DEV) for t in _rand(32, 64, 64, torch.bfloat16, seed=1))
    with pytest.raises(ValueError):
        fused_gated_linear(X, Wg, Wu[:, :32], bg, bu)
    with pytest.raises(ValueError):
        fused_gated_linear(X, Wg, Wu.half(), bg, bu)
    # Forced tensor-core variant on rows TMA cannot address.
    Xo = torch.zeros(32, 65, dtype=torch.bfloat16, device=DEV)[:, :64]
    with pytest.raises(nat.NativeError):
        fused_gated_linear(Xo, Wg, Wu, bg, bu, kernel="umma")


def test_two_layer_ffn_chain():
    g = torch.Generator().manual_seed(17)
    M, K, H = 96, 256, 512
    X = torch.randn(M, K, generator=g).bfloat16()
    W1 = (torch.randn(K, H, generator=g) / K ** 0.5).bfloat16()
    b1 = (torch.rand(H, generator=g) * 0.2 - 0.1).bfloat16()
    W2 = (torch.randn(H, K, generator=g) / H ** 0.5).bfloat16()
    b2 = (torch.rand(K, generator=g) * 0.2 - 0.1).bfloat16()
    ref = oracle.fused_linear_f64(oracle.fused_linear_f64(X, W1, b1, "relu"), W2, b2, None)
    Y = two_layer_ffn(*(t.to(DEV) for t in (X, W1, b1, W2, b2)), "relu")
    _assert_close(Y, ref, torch.bfloat16, "ffn_two_layer")


def test_gated_k_zero_is_act_of_bias_times_bias():
    """K = 0: X Wg and X Wu are zero, so Y = act(bg) * bu (the SIMT path)."""
    M, N = 5, 40
    bg = (torch.rand(N) * 0.2 - 0.1).bfloat16()
    bu = (torch.rand(N) * 0.2 - 0.1).bfloat16()
    X = torch.empty(M, 0, dtype=torch.bfloat16, device=DEV)
    W = torch.empty(0, N, dtype=torch.bfloat16, device=DEV)
    Y = fused_gated_linear(X, W, W, bg.to(DEV), bu.to(DEV), "silu")
    torch.cuda.synchronize()
    assert nat.last_launch_plan().startswith("simt_gated")
    ref = oracle.activation_f64(bg.double().numpy(), "silu") * bu.double().numpy()
    _assert_close(Y, np.broadcast_to(ref, (M, N)), torch.bfloat16, "K=0")
