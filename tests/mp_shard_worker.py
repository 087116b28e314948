"""Worker for tests/test_gpu_multi.py: one process per GPU under torchrun.

Checks, on every rank, the sharded engine against the single-GPU engine on
the same seeded inputs: the column-parallel layer (gathered), the
column -> row MLP and the column -> row gated FFN, each with the NVLink
reduce-broadcast and with NCCL.  Exits non-zero on a mismatch.
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from deepx_op_gpukernelcompiler_b200 import (_native, fused_linear, gated_ffn,  # noqa: E402
                                             mlp_residual)
from deepx_op_gpukernelcompiler_b200.shard import (ColumnParallelLinear,  # noqa: E402
                                                   ParallelGatedFFN, ParallelMLP)


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    failures = []
    try:
        g = torch.Generator(device=dev)
        g.manual_seed(7)
        M, K, N = 1024, 1024, 2560
        X = torch.randn(M, K, generator=g, device=dev).bfloat16()
        W = (torch.randn(K, N, generator=g, device=dev) / K ** 0.5).bfloat16()
        b = (torch.rand(N, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
        full = fused_linear(X, W, b, "silu").float()
        col = ColumnParallelLinear(W, b, "silu", gather_output=True)
        got = col(X).float()
        torch.cuda.synchronize()
        # A shard may be scheduled with a different K split of its last tiles
        # than the full problem, so compare within the bf16 tolerance.
        err = (got - full).abs()
        if bool((err > 2e-2 + 2e-2 * full.abs()).any()):
            failures.append(f"column-parallel differs: max {err.max().item():.4g}")

        H = 4096
        W1 = (torch.randn(K, H, generator=g, device=dev) / K ** 0.5).bfloat16()
        b1 = (torch.rand(H, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
        W2 = (torch.randn(H, K, generator=g, device=dev) / H ** 0.5).bfloat16()
        b2 = (torch.rand(K, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
        ref = mlp_residual(X, W1, b1, W2, b2, "gelu").float()
        for mode, chunks in (("nccl", 1), ("nccl", 4), ("fused", 1)):
            mlp = ParallelMLP(W1, b1, W2, b2, "gelu", chunks=chunks, mode=mode)
            for rep in range(2):  # the fused mode reuses its peer buffers
                out = mlp(X).float()
                torch.cuda.synchronize()
                err = (out - ref).abs()
                tol = 2e-2 + 2e-2 * ref.abs()
                if bool((err > tol).any()):
                    failures.append(f"MLP ({mode}, chunks={chunks}, call {rep}) off by up to "
                                    f"{err.max().item():.4g}")

        Wg = (torch.randn(K, H, generator=g, device=dev) / K ** 0.5).bfloat16()
        Wu = (torch.randn(K, H, generator=g, device=dev) / K ** 0.5).bfloat16()
        bg = (torch.rand(H, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
        bu = (torch.rand(H, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
        ref = gated_ffn(X, Wg, bg, Wu, bu, W2, b2, "silu").float()
        for mode in ("nccl", "fused"):
            ffn = ParallelGatedFFN(Wg, bg, Wu, bu, W2, b2, "silu", mode=mode)
            for rep in range(2):
                out = ffn(X).float()
                torch.cuda.synchronize()
                err = (out - ref).abs()
                if bool((err > 2e-2 + 2e-2 * ref.abs()).any()):
                    failures.append(f"gated FFN ({mode}, call {rep}) off by up to "
                                    f"{err.max().item():.4g}")
        status = _native.device_status(torch.cuda.current_stream(dev).cuda_stream)
        if status:
            failures.append(f"device status {status}")
    finally:
        dist.barrier()
        dist.destroy_process_group()
    for f in failures:
        print(f"rank {rank}/{world}: {f}", flush=True)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
