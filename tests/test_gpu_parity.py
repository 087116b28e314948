"""Engine parity on the GPU, through the C ABI (gpu).

Every kernel variant against the golden outputs of the reference oracle and
against the CPU oracle on seeded inputs, at the tolerances of the workloads:
fp32 rtol = atol = 1e-4, fp16/bf16 (fp32 accumulate) rtol = atol = 2e-2.
"""
import numpy as np
import pytest
import torch

import oracle
from deepx_op_gpukernelcompiler_b200 import _native as nat
from deepx_op_gpukernelcompiler_b200 import fused_linear, mlp_residual
from deepx_op_gpukernelcompiler_b200.linear import selected_kernel
from golden_data import cases, load

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-4, 1e-4), torch.float16: (2e-2, 2e-2), torch.bfloat16: (2e-2, 2e-2)}
DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
DEV = torch.device("cuda:0")


def _variants(case):
    if case["dtype"] == "f32":
        return ["auto", "simt"]
    out = ["auto", "simt", "umma", "umma_1cta"]
    if case["M"] <= 64:
        out.append("decode")
    return out


def _assert_close(got: torch.Tensor, ref, dtype, what=""):
    rtol, atol = TOL[dtype]
    g = got.float().cpu().numpy()
    r = ref.numpy() if isinstance(ref, torch.Tensor) else np.asarray(ref)
    bad = ~np.isclose(g, r, rtol=rtol, atol=atol)
    if bad.any():
        idx = np.argwhere(bad)[0]
        raise AssertionError(f"{what}: {bad.sum()} of {bad.size} elements off; first at {tuple(idx)}: "
                             f"got {g[tuple(idx)]}, want {r[tuple(idx)]}; max |diff| "
                             f"{np.abs(g - r).max():.4g}")


def _status_clean():
    assert nat.device_status(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize("case", [c for c in cases() if not c["mlp"] and not c.get("gated")],
                         ids=lambda c: c["name"])
def test_golden_linear(case):
    t = {k: v.to(DEV) for k, v in load(case).items()}
    dt = DT[case["dtype"]]
    for kern in _variants(case):
        Y = fused_linear(t["X"], t["W"], t["bias"], case["act"], residual=t.get("R"), kernel=kern)
        torch.cuda.synchronize()
        _assert_close(Y, t["Y"].cpu(), dt, f"{case['name']} [{kern}]")
    _status_clean()


@pytest.mark.parametrize("case", [c for c in cases() if c["mlp"]], ids=lambda c: c["name"])
def test_golden_mlp(case):
    t = {k: v.to(DEV) for k, v in load(case).items()}
    Y = mlp_residual(t["X"], t["W1"], t["b1"], t["W2"], t["b2"], case["act"])
    torch.cuda.synchronize()
    _assert_close(Y, t["Y"].cpu(), DT[case["dtype"]], case["name"])


def _rand(M, K, N, dtype, seed, residual=False):
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(M, K, generator=g).to(dtype)
    W = (torch.randn(K, N, generator=g) / max(K, 1) ** 0.5).to(dtype)
    b = (torch.rand(N, generator=g) * 0.2 - 0.1).to(dtype)
    R = torch.randn(M, N, generator=g).to(dtype) if residual else None
    return X, W, b, R


SHAPES = [  # (M, K, N): tile edges, ragged K/N/M, single rows/columns
    (1, 64, 128), (7, 72, 136), (16, 1024, 1024), (33, 200, 264), (64, 4096, 512),
    (65, 64, 64), (127, 128, 128), (128, 64, 256), (129, 136, 392), (255, 520, 520),
    (256, 64, 1024), (300, 1000, 8), (513, 256, 760), (1024, 2048, 768),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K,N", SHAPES)
def test_shapes_all_variants(M, K, N, dtype):
    X, W, b, _ = _rand(M, K, N, dtype, seed=M * 7 + K * 3 + N)
    ref = oracle.fused_linear_f64(X, W, b, "gelu_erf")
    Xd, Wd, bd = X.to(DEV), W.to(DEV), b.to(DEV)
    variants = ["auto", "umma", "umma_1cta", "simt"] + (["decode"] if M <= 64 else [])
    for kern in variants:
        Y = fused_linear(Xd, Wd, bd, "gelu_erf", kernel=kern)
        torch.cuda.synchronize()
        _assert_close(Y, ref, dtype, f"{M}x{K}x{N} {dtype} [{kern}]")
    _status_clean()


@pytest.mark.parametrize("act", [None, "relu", "gelu", "gelu_erf", "silu", "swish"])
@pytest.mark.parametrize("kern", ["umma", "umma_1cta", "decode"])
def test_activations_with_residual(act, kern):
    M = 48 if kern == "decode" else 600
    X, W, b, R = _rand(M, 256, 320, torch.bfloat16, seed=11, residual=True)
    ref = oracle.fused_linear_f64(X, W, b, act, residual=R)
    Y = fused_linear(X.to(DEV), W.to(DEV), b.to(DEV), act, residual=R.to(DEV), kernel=kern)
    torch.cuda.synchronize()
    _assert_close(Y, ref, torch.bfloat16, f"{act} residual [{kern}]")


@pytest.mark.parametrize("kern", ["umma", "umma_1cta", "decode", "simt"])
def test_no_bias(kern):
    X, W, _, _ = _rand(32, 128, 256, torch.float16, seed=5)
    ref = oracle.fused_linear_f64(X, W, None, "relu")
    Y = fused_linear(X.to(DEV), W.to(DEV), None, "relu", kernel=kern)
    torch.cuda.synchronize()
    _assert_close(Y, ref, torch.float16, f"no bias [{kern}]")


@pytest.mark.parametrize("kern,M", [("umma", 300), ("umma_1cta", 40), ("decode", 40),
                                    ("simt", 40)])
def test_strided_views(kern, M):
    """Row pitches larger than the row length (column slices of wider buffers)."""
    K, N = 192, 256
    X, W, b, R = _rand(M, K, N, torch.bfloat16, seed=9, residual=True)
    Xb = torch.zeros(M, K + 64, dtype=X.dtype)
    Xb[:, 32:32 + K] = X
    Wb = torch.zeros(K, N + 128, dtype=W.dtype)
    Wb[:, 64:64 + N] = W
    Rb = torch.zeros(M, N + 8, dtype=R.dtype)
    Rb[:, :N] = R
    Xd, Wd, Rd = Xb.to(DEV), Wb.to(DEV), Rb.to(DEV)
    Yb = torch.full((M, N + 16), 7.0, dtype=X.dtype, device=DEV)
    out = Yb[:, 8:8 + N]
    fused_linear(Xd[:, 32:32 + K], Wd[:, 64:64 + N], b.to(DEV), "silu", residual=Rd[:, :N],
                 out=out, kernel=kern)
    torch.cuda.synchronize()
    ref = oracle.fused_linear_f64(X, W, b, "silu", residual=R)
    _assert_close(out, ref, torch.bfloat16, f"strided [{kern}]")
    assert torch.all(Yb[:, :8] == 7) and torch.all(Yb[:, 8 + N:] == 7), "wrote outside out"


def test_fp32_exact_path():
    X, W, b, R = _rand(130, 300, 70, torch.float32, seed=3, residual=True)
    Y = fused_linear(X.to(DEV), W.to(DEV), b.to(DEV), "gelu", residual=R.to(DEV))
    torch.cuda.synchronize()
    _assert_close(Y, oracle.fused_linear_f64(X, W, b, "gelu", residual=R), torch.float32, "fp32")


def test_misaligned_rows_fall_back_to_simt():
    """K = 45: rows are not 16-byte multiples, so TMA cannot address them."""
    X, W, b, _ = _rand(100, 45, 77, torch.bfloat16, seed=4)
    assert selected_kernel(100, 77, 45, torch.bfloat16) == "simt"
    Y = fused_linear(X.to(DEV), W.to(DEV), b.to(DEV), "relu")
    torch.cuda.synchronize()
    _assert_close(Y, oracle.fused_linear_f64(X, W, b, "relu"), torch.bfloat16, "K=45 auto")
    with pytest.raises(nat.NativeError) as ei:
        fused_linear(X.to(DEV), W.to(DEV), b.to(DEV), "relu", kernel="umma")
    assert ei.value.code == nat.DX_ERR_UNSUPPORTED


def test_k_zero_gives_act_of_bias():
    b = torch.tensor([1.0, -2.0, 3.0, -4.0] * 4, dtype=torch.bfloat16)
    X = torch.empty(5, 0, dtype=torch.bfloat16, device=DEV)
    W = torch.empty(0, 16, dtype=torch.bfloat16, device=DEV)
    Y = fused_linear(X, W, b.to(DEV), "relu")
    torch.cuda.synchronize()
    assert torch.equal(Y.cpu(), torch.relu(b).expand(5, 16))


@pytest.mark.parametrize("M", [1, 4, 16])
def test_whole_tile_decode_needs_no_workspace(M):
    """With at least half as many 256-column tiles as SMs the decode kernel
    streams one whole tile per CTA and needs no workspace: AUTO picks it even
    when the caller passes none (M = 1 included)."""
    lib = nat.load()
    K, N = 1024, 28672
    X, W, b, _ = _rand(M, K, N, torch.float16, seed=M)
    Xd, Wd, bd = X.to(DEV), W.to(DEV), b.to(DEV)
    Y = torch.empty(M, N, dtype=torch.float16, device=DEV)
    assert lib.dx_fused_linear_workspace_size(M, N, K, nat.DX_DTYPE_F16, nat.DX_KERNEL_DECODE) == 0
    rc = lib.dx_fused_linear(Xd.data_ptr(), Wd.data_ptr(), bd.data_ptr(), None, Y.data_ptr(),
                             M, N, K, K, N, 0, N, nat.DX_DTYPE_F16, nat.DX_ACT_GELU_ERF, None, 0,
                             None)
    assert rc == nat.DX_OK, nat.last_error()
    assert nat.last_launch_plan().startswith("decode"), nat.last_launch_plan()
    torch.cuda.synchronize()
    _assert_close(Y, oracle.fused_linear_f64(X, W, b, "gelu_erf"), torch.float16, f"M={M}")
    _status_clean()


def test_decode_without_workspace_is_rejected():
    lib = nat.load()
    X, W, b, _ = _rand(16, 128, 256, torch.float16, seed=1)
    Xd, Wd, bd = X.to(DEV), W.to(DEV), b.to(DEV)
    Y = torch.empty(16, 256, dtype=torch.float16, device=DEV)
    rc = lib.dx_fused_linear_ex(Xd.data_ptr(), Wd.data_ptr(), bd.data_ptr(), None, Y.data_ptr(),
                                16, 256, 128, 128, 256, 0, 256, nat.DX_DTYPE_F16, 0,
                                nat.DX_KERNEL_DECODE, None, 0, None)
    assert rc == nat.DX_ERR_WORKSPACE
    # AUTO without a workspace picks the tensor-core GEMM instead.
    rc = lib.dx_fused_linear(Xd.data_ptr(), Wd.data_ptr(), bd.data_ptr(), None, Y.data_ptr(),
                             16, 256, 128, 128, 256, 0, 256, nat.DX_DTYPE_F16, 0, None, 0, None)
    assert rc == nat.DX_OK
    torch.cuda.synchronize()
    _assert_close(Y, oracle.fused_linear_f64(X, W, b, None), torch.float16, "auto w/o workspace")


@pytest.mark.parametrize("kern,M", [("umma", 1000), ("umma_1cta", 1000), ("decode", 16)])
def test_bitwise_deterministic(kern, M):
    X, W, b, _ = _rand(M, 2048, 1536, torch.bfloat16, seed=21)
    Xd, Wd, bd = X.to(DEV), W.to(DEV), b.to(DEV)
    Y1 = fused_linear(Xd, Wd, bd, "silu", kernel=kern)
    Y2 = fused_linear(Xd, Wd, bd, "silu", kernel=kern)
    torch.cuda.synchronize()
    assert torch.equal(Y1, Y2)


def test_decode_tickets_reset_across_shapes():
    """The split-K workspace is reused across calls of different shapes: the
    partial sums of a narrow problem must not land on the tickets a wider
    problem uses later (24 n-tiles, then 8, then 24 again)."""
    for (M, K, N) in [(16, 4096, 3072), (16, 4096, 1024), (3, 640, 2048), (64, 8192, 256),
                      (16, 8192, 3072), (16, 1024, 3072), (16, 4096, 1024)]:
        X, W, b, _ = _rand(M, K, N, torch.float16, seed=M + K + N)
        Y = fused_linear(X.to(DEV), W.to(DEV), b.to(DEV), "gelu_erf", kernel="decode")
        torch.cuda.synchronize()
        _assert_close(Y, oracle.fused_linear_f64(X, W, b, "gelu_erf"), torch.float16,
                      f"decode {M}x{K}x{N}")
    _status_clean()



@pytest.mark.parametrize("M,K,N", [(16, 8192, 3584), (3, 4096, 1024), (16, 2048, 512)])
def test_decode_fixup_bitwise_across_repeats(M, K, N):
    """The last CTA to reach a split tile sums the partials either from bulk
    copies staged in shared memory (when the tile is its last work item, in
    batches when the tile has many segments) or from registers.  Both add in
    the same fixed segment order, so repeats whose arrival order differs
    agree to the last bit (M = 3: only the first rows are staged)."""
    X, W, b, _ = _rand(M, K, N, torch.float16, seed=M + N)
    Xd, Wd, bd = X.to(DEV), W.to(DEV), b.to(DEV)
    Y0 = fused_linear(Xd, Wd, bd, "gelu_erf", kernel="decode")
    assert "grid=" in nat.last_launch_plan()
    for rep in range(6):
        Y = fused_linear(Xd, Wd, bd, "gelu_erf", kernel="decode")
        assert torch.equal(Y, Y0), f"repeat {rep} differs"
    torch.cuda.synchronize()
    _assert_close(Y0, oracle.fused_linear_f64(X, W, b, "gelu_erf"), torch.float16,
                  f"decode {M}x{K}x{N}")
    _status_clean()


@pytest.mark.parametrize("kern,M", [("decode", 16), ("umma", 256)])
@pytest.mark.parametrize("act", ["gelu_erf", "gelu", "silu"])
def test_activation_accuracy_across_range(kern, M, act):
    """Y = act(X W + b) with W = I, so each output is act(x) of one fp16
    input, x over [-12, 12].  GELU-erf (published erfc approximation) is
    within one fp16 ulp of the fp64 value, or 1e-6 where the value is that
    small.  GELU-tanh and SiLU take the hardware tanh (relative error about
    2^-11 of tanh, so up to 2.5e-4 |x| absolute where 1 + tanh cancels)."""
    K = N = 256
    x = torch.linspace(-12.0, 12.0, M * K).reshape(M, K).to(torch.float16)
    W = torch.zeros(K, N, dtype=torch.float16)
    W[torch.arange(K), torch.arange(K)] = 1.0
    b = torch.zeros(N, dtype=torch.float16)
    Y = fused_linear(x.to(DEV), W.to(DEV), b.to(DEV), act, kernel=kern)
    torch.cuda.synchronize()
    v = x.double()
    if act == "gelu_erf":
        ref = 0.5 * v * torch.special.erfc(-v / 2 ** 0.5)
    elif act == "gelu":
        ref = 0.5 * v * (1 + torch.tanh((2 / torch.pi) ** 0.5 * (v + 0.044715 * v ** 3)))
    else:
        ref = v * torch.sigmoid(v)
    got = Y.cpu().double()
    ulp = torch.finfo(torch.float16).eps * ref.abs().clamp_min(2.0 ** -14)
    err = (got - ref).abs()
    if act == "gelu_erf":
        bad = (err > ulp) & (err > 1e-6)
    else:
        bad = err > ulp + 2.5e-4 * v.abs()
    assert not bad.any(), (f"{act} [{kern}]: {int(bad.sum())} off, e.g. x={float(v[bad][0]):.4f} "
                           f"got {float(got[bad][0]):.6g} want {float(ref[bad][0]):.6g}")

def test_nonzero_stream():
    s = torch.cuda.Stream()
    X, W, b, _ = _rand(256, 512, 512, torch.bfloat16, seed=2)
    with torch.cuda.stream(s):
        Y = fused_linear(X.to(DEV), W.to(DEV), b.to(DEV), "relu")
    s.synchronize()
    _assert_close(Y, oracle.fused_linear_f64(X, W, b, "relu"), torch.bfloat16, "side stream")


def _call_abi(X, W, b, R, act, kernel, workspace):
    """dx_fused_linear_ex with an explicit workspace (None: whole tiles only)."""
    lib = nat.load()
    M, K = X.shape
    N = W.shape[1]
    Y = torch.empty(M, N, dtype=X.dtype, device=DEV)
    ws_ptr = workspace.data_ptr() if workspace is not None else None
    ws_len = workspace.numel() if workspace is not None else 0
    rc = lib.dx_fused_linear_ex(X.data_ptr(), W.data_ptr(), b.data_ptr(),
                                R.data_ptr() if R is not None else None, Y.data_ptr(),
                                M, N, K, K, N, N if R is not None else 0, N,
                                nat.DX_DTYPE_BF16 if X.dtype == torch.bfloat16 else nat.DX_DTYPE_F16,
                                {"gelu": nat.DX_ACT_GELU_TANH, "silu": nat.DX_ACT_SILU}[act],
                                nat.KERNEL_NAMES[kernel], ws_ptr, ws_len,
                                torch.cuda.current_stream().cuda_stream)
    nat.check("dx_fused_linear_ex", rc)
    return Y, nat.last_launch_plan()


@pytest.mark.parametrize("M,N", [(256, 128), (512, 512), (768, 1280), (1280, 384)])
def test_pair_and_single_cta_agree(M, N):
    """Without a workspace (whole tiles only) the CTA-pair and single-CTA
    kernels accumulate in the same k order, so they agree to the last bit."""
    X, W, b, R = _rand(M, 1024, N, torch.bfloat16, seed=M + N, residual=True)
    Xd, Wd, bd, Rd = X.to(DEV), W.to(DEV), b.to(DEV), R.to(DEV)
    Y2, plan2 = _call_abi(Xd, Wd, bd, Rd, "gelu", "umma", None)
    Y1, plan1 = _call_abi(Xd, Wd, bd, Rd, "gelu", "umma_1cta", None)
    torch.cuda.synchronize()
    assert "splits=1" in plan2 and "splits=1" in plan1
    _assert_close(Y2, oracle.fused_linear_f64(X, W, b, "gelu", residual=R), torch.bfloat16,
                  f"pair {M}x{N}")
    assert torch.equal(Y1, Y2)


SPLIT_SHAPES = [  # (M, K, N): a partial last wave of tiles, K long enough to split
    (8192, 4096, 1792), (1024, 4096, 1792), (512, 2048, 640), (300, 1024, 264), (4096, 4096, 4096),
    (2048, 8192, 1024),
]
# Shapes whose plan must split (the planner may prefer whole tiles elsewhere).
MUST_SPLIT = {(8192, 4096, 1792), (512, 2048, 640), (4096, 4096, 4096)}


@pytest.mark.parametrize("kern", ["umma", "umma_1cta"])
@pytest.mark.parametrize("M,K,N", SPLIT_SHAPES)
def test_split_tail(M, K, N, kern):
    """Tiles of the last partial wave are split along K over idle SMs; the
    partial sums are reduced in fixed order, so results are deterministic and
    match the oracle."""
    X, W, b, R = _rand(M, K, N, torch.bfloat16, seed=M + 3 * N, residual=True)
    Xd, Wd, bd, Rd = X.to(DEV), W.to(DEV), b.to(DEV), R.to(DEV)
    ws = torch.zeros(nat.load().dx_fused_linear_workspace_size(M, N, K, nat.DX_DTYPE_BF16,
                                                               nat.KERNEL_NAMES[kern]),
                     dtype=torch.uint8, device=DEV)
    Ya, plan = _call_abi(Xd, Wd, bd, Rd, "silu", kern, ws)
    Yb, _ = _call_abi(Xd, Wd, bd, Rd, "silu", kern, ws)
    torch.cuda.synchronize()
    if (M, K, N) in MUST_SPLIT:
        assert "splits=1 " not in plan, plan
    ref = oracle.fused_linear_f32(X, W, b, "silu", residual=R) if M * N * K > 2**31 else \
        oracle.fused_linear_f64(X, W, b, "silu", residual=R)
    _assert_close(Ya, ref, torch.bfloat16, f"split {M}x{K}x{N} [{kern}] {plan}")
    assert torch.equal(Ya, Yb), "split reduction is not deterministic"
    assert int(ws[:65536].view(torch.int32).abs().sum().item()) == 0, "tickets not reset"
    _status_clean()


@pytest.mark.parametrize("M,K,N,blocks", [(8192, 4096, 14336, (2, 4)), (8192, 4096, 14336, (8, 8)),
                                           (300, 136, 1000, (3, 5)),
                                           (1, 64, 520, (1, 2)), (513, 256, 760, (2, 3))])
def test_host_entry_matches_device_entry(M, K, N, blocks):
    """fused_linear_host (blocks copied in and out around per-block launches)
    gives the device entry's result; unpinned and pinned host memory."""
    from deepx_op_gpukernelcompiler_b200 import fused_linear_host
    X, W, b, _ = _rand(M, K, N, torch.bfloat16, seed=M + N)
    ref = fused_linear(X.to(DEV), W.to(DEV), b.to(DEV), "silu").float().cpu()
    for pinned in (True, False):
        Xh, Wh, bh = (t.pin_memory() if pinned else t for t in (X, W, b))
        out = torch.empty(M, N, dtype=torch.bfloat16)
        if pinned:
            out = out.pin_memory()
        fused_linear_host(Xh, Wh, bh, "silu", out=out, device=DEV, row_blocks=blocks[0],
                          col_blocks=blocks[1])
        torch.cuda.synchronize()
        _assert_close(out, ref, torch.bfloat16, f"host {M}x{K}x{N} pinned={pinned}")
    # No bias, default blocks, output allocated by the call.
    out = fused_linear_host(X, W, None, None, device=DEV)
    torch.cuda.synchronize()
    ref_nb = fused_linear(X.to(DEV), W.to(DEV), None, None).float().cpu()
    _assert_close(out, ref_nb, torch.bfloat16, "host, no bias")


def test_bounded_wait_reports_timeout_and_context_survives():
    """A wait that nothing completes gives up after its bound (about a second),
    sets DX_DEVICE_STATUS_TIMEOUT and returns; the next launches run normally."""
    lib = nat.load()
    stream = torch.cuda.current_stream().cuda_stream
    assert nat.device_status(stream) == 0
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    nat.check("dx_selftest_bounded_wait", lib.dx_selftest_bounded_wait(flag.data_ptr(), stream))
    assert nat.device_status(stream) == nat.DX_DEVICE_STATUS_TIMEOUT
    assert flag.item() == 2
    assert nat.device_status(stream) == 0  # read-and-clear
    X, W, b, _ = _rand(300, 256, 512, torch.bfloat16, seed=77)
    Y = fused_linear(X.to(DEV), W.to(DEV), b.to(DEV), "silu")
    torch.cuda.synchronize()
    _assert_close(Y, oracle.fused_linear_f64(X, W, b, "silu"), torch.bfloat16, "after timeout")
    _status_clean()


def test_timeout_makes_the_next_call_raise():
    """A launch whose bounded wait ran out is reported by the next call on
    the device (through the status word's host-mapped copy, no added
    synchronisation): fused_linear raises DX_ERR_DEVICE_TIMEOUT until
    dx_device_status has read and cleared the condition."""
    lib = nat.load()
    stream = torch.cuda.current_stream().cuda_stream
    assert nat.device_status(stream) == 0
    X, W, b, _ = _rand(300, 256, 512, torch.bfloat16, seed=78)
    Xd, Wd, bd = X.to(DEV), W.to(DEV), b.to(DEV)
    fused_linear(Xd, Wd, bd, "silu")  # installs the host-mapped copy on this device
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    nat.check("dx_selftest_bounded_wait", lib.dx_selftest_bounded_wait(flag.data_ptr(), stream))
    torch.cuda.synchronize()  # the wait has given up by now
    with pytest.raises(nat.NativeError) as info:
        fused_linear(Xd, Wd, bd, "silu")
    assert info.value.code == nat.DX_ERR_DEVICE_TIMEOUT
    assert "bounded wait" in str(info.value)
    assert nat.device_status(stream) == nat.DX_DEVICE_STATUS_TIMEOUT  # read and clear
    Y = fused_linear(Xd, Wd, bd, "silu")
    torch.cuda.synchronize()
    _assert_close(Y, oracle.fused_linear_f64(X, W, b, "silu"), torch.bfloat16, "after clear")
    _status_clean()


def test_loaded_kernels_are_sm100a():
    """The kernels the driver loaded from the library are SASS for sm_100
    (binaryVersion 100), with no PTX that could be JIT-compiled instead."""
    import ctypes
    binv, ptxv = ctypes.c_int(0), ctypes.c_int(-1)
    nat.check("dx_kernel_arch", nat.load().dx_kernel_arch(ctypes.byref(binv), ctypes.byref(ptxv)))
    assert binv.value == 100
    assert ptxv.value in (0, 100)


@pytest.mark.parametrize("M,K,N,cluster", [(16, 8192, 3584, 8), (16, 4096, 7168, 4),
                                           (16, 2048, 14336, 2), (5, 2048, 3072, 8),
                                           (24, 2048, 3584, 8), (48, 1024, 3584, 8)])
def test_decode_cluster_split(M, K, N, cluster):
    """Fewer 256-column tiles than SMs / 2: each tile's K range is split over
    a thread-block cluster whose CTAs add their partials through distributed
    shared memory — no workspace, deterministic (rank order), every row
    template (M = 5 / 16 / 24 / 48), residual included."""
    lib = nat.load()
    assert lib.dx_fused_linear_workspace_size(M, N, K, nat.DX_DTYPE_F16, nat.DX_KERNEL_DECODE) == 0
    X, W, b, R = _rand(M, K, N, torch.float16, seed=M + K + N, residual=True)
    Xd, Wd, bd, Rd = X.to(DEV), W.to(DEV), b.to(DEV), R.to(DEV)
    Y0 = fused_linear(Xd, Wd, bd, "gelu_erf", residual=Rd, kernel="decode")
    plan = nat.last_launch_plan()
    assert f"cluster={cluster} " in plan and "workspace=0" in plan, plan
    for _ in range(3):
        assert torch.equal(fused_linear(Xd, Wd, bd, "gelu_erf", residual=Rd, kernel="decode"), Y0)
    torch.cuda.synchronize()
    _assert_close(Y0, oracle.fused_linear_f64(X, W, b, "gelu_erf", residual=R), torch.float16,
                  f"cluster decode {M}x{K}x{N} [{plan}]")
    _status_clean()


@pytest.mark.parametrize("kern,M,K", [("decode", 16, 2048), ("decode", 5, 4096), ("umma", 256, 1024),
                                      ("umma_1cta", 256, 1024), ("auto", 16, 2048)])
def test_dependent_launches_back_to_back(kern, M, K):
    """Each launch reads the previous launch's output and overwrites the buffer
    the launch before it read (two buffers, ping-pong), with no host sync in
    between: the GEMM and decode kernels start early (programmatic dependent
    launch) but touch global memory only once the previous grid is complete,
    so the chain must equal, bit for bit, the same chain run with a sync after
    every step; each synced step is checked against the fp64 oracle fed that
    step's device input."""
    g = torch.Generator().manual_seed(M * 7 + K)
    Ws = [(torch.randn(K, K, generator=g) / K ** 0.5).half() for _ in range(2)]
    bs = [(torch.rand(K, generator=g) * 0.2 - 0.1).half() for _ in range(2)]
    X = torch.randn(M, K, generator=g).half()
    Wd, bd = [w.to(DEV) for w in Ws], [b.to(DEV) for b in bs]
    steps = 8

    def chain(sync: bool):
        bufs = [X.to(DEV), torch.empty(M, K, dtype=torch.float16, device=DEV)]
        seen = [X]
        for i in range(steps):
            src, dst = bufs[i % 2], bufs[(i + 1) % 2]
            fused_linear(src, Wd[i % 2], bd[i % 2], "gelu_erf", residual=src, out=dst, kernel=kern)
            if sync:
                torch.cuda.synchronize()
                seen.append(dst.cpu())
        torch.cuda.synchronize()
        return bufs[steps % 2].clone(), seen

    fast, _ = chain(False)
    slow, seen = chain(True)
    assert torch.equal(fast, slow), f"{kern}: back-to-back chain differs from the synced chain"
    for i in range(steps):
        want = oracle.fused_linear_f64(seen[i], Ws[i % 2], bs[i % 2], "gelu_erf", residual=seen[i])
        _assert_close(seen[i + 1], want, torch.float16, f"{kern} chain step {i}")
    _status_clean()


@pytest.mark.parametrize("M,K,N", [(16, 4096, 3584), (16, 2048, 28672)])
def test_weights_written_by_the_previous_launch(M, K, N):
    """A tensor-core launch writes the W that the next (decode) launch reads,
    and the launch after it overwrites that W again, with no host sync: the
    decode kernel must read W only after the producer has completed (its
    early start covers set-up only), and the producer must not overwrite it
    before the decode has read it; bit for bit equal to the synced run."""
    g = torch.Generator().manual_seed(K + N)
    K2 = 512
    A = (torch.randn(K, K2, generator=g) / K2 ** 0.5).half().to(DEV)
    Bs = [(torch.randn(K2, N, generator=g)).half().to(DEV) for _ in range(3)]
    X = torch.randn(M, K, generator=g).half().to(DEV)
    b = (torch.rand(N, generator=g) * 0.2 - 0.1).half().to(DEV)

    def run(sync: bool):
        Wbuf = torch.empty(K, N, dtype=torch.float16, device=DEV)
        outs = []
        for i in range(6):
            fused_linear(A, Bs[i % 3], None, None, out=Wbuf, kernel="umma")  # W of the next step
            if sync:
                torch.cuda.synchronize()
            outs.append(fused_linear(X, Wbuf, b, "gelu_erf", kernel="decode"))
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return outs, Wbuf.cpu()

    fast, _ = run(False)
    slow, W_last = run(True)
    for i, (a, c) in enumerate(zip(fast, slow)):
        assert torch.equal(a, c), f"step {i}: decode read a W its producer had not finished"
    ref = oracle.fused_linear_f64(X.cpu(), W_last, b.cpu(), "gelu_erf")
    _assert_close(slow[5], ref, torch.float16, "decode on a produced W")
    _status_clean()
