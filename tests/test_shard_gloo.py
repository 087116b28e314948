"""Multi-rank partitioning logic on CPU ranks (gloo, world size 2 and 3).

The compute function is the CPU oracle (injected), so what is tested is the
sharding itself: slice bounds, which rank adds b2 and the residual, the
all-reduce, M-chunking and the optional all-gather.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from deepx_op_gpukernelcompiler_b200.shard import (ColumnParallelLinear, ParallelGatedFFN,
                                                   ParallelMLP, shard_bounds)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_linear(X, W, bias=None, activation=None, residual=None, out=None):
    Y = torch.from_numpy(oracle.fused_linear_f64(X, W, bias, activation, residual=residual))
    Y = Y.to(X.dtype)
    if out is not None:
        out.copy_(Y)
        return out
    return Y


def oracle_gated(X, Wg, Wu, bg=None, bu=None, activation="silu", out=None):
    Y = torch.from_numpy(oracle.gated_linear_f64(X, Wg, bg, Wu, bu, activation)).to(X.dtype)
    if out is not None:
        out.copy_(Y)
        return out
    return Y


def _gated_inputs(M=24, K=40, H=200, seed=1):
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(M, K, generator=g, dtype=torch.float64)
    Wg = torch.randn(K, H, generator=g, dtype=torch.float64) / K ** 0.5
    Wu = torch.randn(K, H, generator=g, dtype=torch.float64) / K ** 0.5
    bg = torch.rand(H, generator=g, dtype=torch.float64) * 0.2 - 0.1
    bu = torch.rand(H, generator=g, dtype=torch.float64) * 0.2 - 0.1
    Wo = torch.randn(H, K, generator=g, dtype=torch.float64) / H ** 0.5
    bo = torch.rand(K, generator=g, dtype=torch.float64) * 0.2 - 0.1
    return X, Wg, bg, Wu, bu, Wo, bo


def _inputs(M=24, K=40, H=200, seed=0):
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(M, K, generator=g, dtype=torch.float64)
    W1 = torch.randn(K, H, generator=g, dtype=torch.float64) / K ** 0.5
    b1 = torch.rand(H, generator=g, dtype=torch.float64) * 0.2 - 0.1
    W2 = torch.randn(H, K, generator=g, dtype=torch.float64) / H ** 0.5
    b2 = torch.rand(K, generator=g, dtype=torch.float64) * 0.2 - 0.1
    return X, W1, b1, W2, b2


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        X, W1, b1, W2, b2 = _inputs()
        col = ColumnParallelLinear(W1, b1, "silu", linear_fn=oracle_linear, align=8)
        Y_local = col(X)
        col_g = ColumnParallelLinear(W1, b1, "silu", linear_fn=oracle_linear, align=8,
                                     gather_output=True)
        Y_full = col_g(X)
        mlp = ParallelMLP(W1, b1, W2, b2, "gelu", linear_fn=oracle_linear, chunks=3, align=8)
        Y_mlp = mlp(X)
        Xg, Wg, bg, Wu, bu, Wo, bo = _gated_inputs()
        ffn = ParallelGatedFFN(Wg, bg, Wu, bu, Wo, bo, "silu", gated_fn=oracle_gated,
                               linear_fn=oracle_linear, chunks=2, align=8)
        Y_gated = ffn(Xg)
        results[rank] = {"n0": col.n0, "n1": col.n1, "Y_local": Y_local.numpy(),
                         "Y_full": Y_full.numpy(), "Y_mlp": Y_mlp.numpy(),
                         "Y_gated": Y_gated.numpy(), "gated_mode": ffn.mode}
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_column_and_mlp_sharding(world):
    port = _free_port()
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_worker, args=(world, port, results), nprocs=world, join=True,
                           start_method="spawn")
        res = dict(results)
    X, W1, b1, W2, b2 = _inputs()
    full = oracle.fused_linear_f64(X, W1, b1, "silu")
    mlp = oracle.mlp_residual_f64(X, W1, b1, W2, b2, "gelu")
    gated = oracle.gated_ffn_f64(*_gated_inputs(), act="silu")
    covered = []
    for r in range(world):
        n0, n1 = res[r]["n0"], res[r]["n1"]
        covered.append((n0, n1))
        np.testing.assert_allclose(res[r]["Y_local"], full[:, n0:n1], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(res[r]["Y_full"], full, rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(res[r]["Y_mlp"], mlp, rtol=1e-10, atol=1e-10)
        np.testing.assert_allclose(res[r]["Y_gated"], gated, rtol=1e-10, atol=1e-10)
        assert res[r]["gated_mode"] == "nccl"
    assert covered[0][0] == 0 and covered[-1][1] == W1.shape[1]
    assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))


@pytest.mark.parametrize("n,world,align", [(14336, 8, 64), (16384, 8, 64), (200, 3, 8),
                                           (100, 4, 64), (7, 2, 1), (1792, 3, 128)])
def test_shard_bounds_partition(n, world, align):
    bounds = [shard_bounds(n, world, r, align) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == n
    for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
        assert a1 == b0
    for s, e in bounds:
        assert s % align == 0 or s == n
    sizes = [e - s for s, e in bounds]
    assert max(sizes) - min(sizes) <= align


def test_shard_bounds_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)
