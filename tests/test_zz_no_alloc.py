"""The decode entry point that allocates nothing (gpu).

Some callers cannot allocate device memory when they launch a kernel: a
runtime whose own heap manager owns every device buffer hands the kernel only
raw pointers and a stream, so it has no workspace to pass and may not call
cudaMalloc behind its allocator's back.  ``dx_fused_linear_decode_noalloc``
serves them: it runs the split-K decode kernel with its scratch in a fixed
array inside the library.  Its output must be bitwise equal to the
workspace-taking entry point (``dx_fused_linear`` via
``fused_linear(kernel="decode")``, which runs the same deterministic plan)
and within the fp16/bf16 tolerance of the fp64 oracle, on consecutive calls
that reuse the shared scratch — split-K plans of every row template (16, 32
and 64 padded rows), and plans that need no scratch (tiles split over a
thread-block cluster, whole tiles).

This file is collected last so that a failure here comes after every other
test has run.
"""
import numpy as np
import pytest
import torch

import oracle
from deepx_op_gpukernelcompiler_b200 import _native as nat
from deepx_op_gpukernelcompiler_b200 import fused_linear

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
RTOL = ATOL = 2e-2  # fp16/bf16 with fp32 accumulation, as in test_gpu_parity
DTYPES = {torch.float16: nat.DX_DTYPE_F16, torch.bfloat16: nat.DX_DTYPE_BF16}
_ACT = {None: nat.DX_ACT_NONE, "relu": nat.DX_ACT_RELU, "gelu_erf": nat.DX_ACT_GELU_ERF,
        "silu": nat.DX_ACT_SILU}


def _inputs(M, K, N, dtype, seed, residual=False):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    X = torch.randn(M, K, generator=g, device=DEV).to(dtype)
    W = (torch.randn(K, N, generator=g, device=DEV) / K ** 0.5).to(dtype)
    b = (torch.rand(N, generator=g, device=DEV) * 0.2 - 0.1).to(dtype)
    R = torch.randn(M, N, generator=g, device=DEV).to(dtype) if residual else None
    return X, W, b, R


def _noalloc(X, W, b, R, act):
    M, K = X.shape
    N = W.shape[1]
    Y = torch.empty(M, N, dtype=X.dtype, device=DEV)
    rc = nat.load().dx_fused_linear_decode_noalloc(
        X.data_ptr(), W.data_ptr(), b.data_ptr(), R.data_ptr() if R is not None else None,
        Y.data_ptr(), M, N, K, K, N, N if R is not None else 0, N, DTYPES[X.dtype],
        _ACT[act], torch.cuda.current_stream(DEV).cuda_stream)
    nat.check("dx_fused_linear_decode_noalloc", rc)
    return Y


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    # Consecutive calls with different shapes share the static scratch; the
    # last repeats the first to show nothing stale carries over.  Every
    # split-K case must fit the 8 MiB array; the whole-tile case needs none.
    lib = nat.load()
    calls = [
        # M, K, N, dtype, act, seed, residual, split-K through the scratch
        (16, 4096, 1536, torch.float16, "gelu_erf", 1, False, True),
        (5, 2048, 1536, torch.bfloat16, "silu", 2, True, True),
        (24, 2048, 1536, torch.float16, "relu", 4, False, True),    # 32-row template
        (48, 1024, 1536, torch.bfloat16, "gelu_erf", 5, True, True),  # 64-row template
        (16, 4096, 3072, torch.float16, "silu", 7, False, False),   # cluster of 8 per tile
        (16, 1024, 28672, torch.float16, "silu", 6, False, False),  # whole tiles
        (16, 4096, 1536, torch.float16, "gelu_erf", 1, False, True),
    ]
    for M, K, N, dtype, act, seed, residual, split in calls:
        need = lib.dx_fused_linear_workspace_size(M, N, K, DTYPES[dtype], nat.DX_KERNEL_DECODE)
        assert (0 < need <= (8 << 20)) if split else need == 0, (M, K, N, need)
        X, W, b, R = _inputs(M, K, N, dtype, seed, residual)
        got = _noalloc(X, W, b, R, act)
        want = fused_linear(X, W, b, act, residual=R, kernel="decode")
        torch.cuda.synchronize()
        assert torch.equal(got, want), (
            f"{M}x{K}x{N} {dtype}: max |diff| {(got.float() - want.float()).abs().max().item()}")
        ref = oracle.fused_linear_f64(X.cpu(), W.cpu(), b.cpu(), act,
                                      residual=R.cpu() if R is not None else None)
        np.testing.assert_allclose(got.float().cpu().numpy(), ref, rtol=RTOL, atol=ATOL,
                                   err_msg=f"{M}x{K}x{N} {dtype} {act} against the fp64 oracle")
    assert nat.device_status(torch.cuda.current_stream(DEV).cuda_stream) == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    # 8 tiles of 256 columns (too few for a cluster to cover half the SMs, so
    # K is split over the SMs through the scratch): up to 19 segments x 64
    # padded rows x 256 columns of fp32 partial sums per tile, 9.6 MiB > the
    # 8 MiB array.
    M, K, N = 64, 8192, 2048
    lib = nat.load()
    assert lib.dx_fused_linear_workspace_size(M, N, K, nat.DX_DTYPE_F16,
                                              nat.DX_KERNEL_DECODE) > (8 << 20)
    X, W, b, _ = _inputs(M, K, N, torch.float16, 3)
    Y = torch.empty(M, N, dtype=torch.float16, device=DEV)
    rc = lib.dx_fused_linear_decode_noalloc(
        X.data_ptr(), W.data_ptr(), b.data_ptr(), None, Y.data_ptr(), M, N, K, K, N,
        0, N, nat.DX_DTYPE_F16, nat.DX_ACT_NONE, torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == nat.DX_ERR_WORKSPACE
    assert "static scratch" in nat.last_error()
