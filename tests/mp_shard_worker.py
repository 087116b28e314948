"""Worker for tests/test_gpu_multi.py: one process per GPU under torchrun.

Checks, on every rank, the sharded engine against the fp64 CPU oracle (the
reference expression act(a @ b + bias), kernel.py:64-66, restated in
oracle/) on row blocks of the same seeded inputs:

* the column-parallel layer (gathered);
* the column -> row MLP, Y = GELU(X W1 + b1) W2 + b2 + X, with the
  overlapped NVLink reduction carried by the GEMM launches (1, 3 and 4 row
  chunks, the first GEMM grouped or not; its NVLink-multicast form where the
  fabric offers it, and its peer-load form) and with NCCL;
* the column -> row gated FFN, both reductions;
* a row count the overlapped reduction cannot take (M not a multiple of the
  world size, as decode rows are): it must run the NCCL path and still be
  right;
* output ownership: a second call must not overwrite the first call's Y.

Bit equality between the two reductions is not expected (NCCL sums in its own
order); each is held to the bf16 tolerance rtol = atol = 2e-2 against the
oracle.  Exits non-zero on any mismatch.
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import oracle  # noqa: E402
from deepx_op_gpukernelcompiler_b200 import _native  # noqa: E402
from deepx_op_gpukernelcompiler_b200.shard import (ColumnParallelLinear,  # noqa: E402
                                                   ParallelGatedFFN, ParallelMLP)

TOL = 2e-2


def row_blocks(M: int, rows: int = 16) -> list[tuple[int, int]]:
    """First, middle (straddling a slab boundary) and last row blocks."""
    mid = max(0, M // 2 - rows // 2)
    blocks = [(0, min(rows, M)), (mid, min(M, mid + rows)), (max(0, M - rows), M)]
    return sorted(set(blocks))


def cpu(t):
    return t.detach().float().cpu().numpy()


def compare(name, got, want_fn, M, failures, blocks=None):
    """got: [M, N] device tensor; want_fn(r0, r1) -> fp64 oracle rows."""
    g = cpu(got)
    worst = 0.0
    for r0, r1 in (blocks or row_blocks(M)):
        want = want_fn(r0, r1)
        err = np.abs(g[r0:r1] - want)
        bad = err > TOL + TOL * np.abs(want)
        worst = max(worst, float(err.max()) if err.size else 0.0)
        if bad.any():
            failures.append(f"{name}: rows {r0}..{r1} off by up to {float(err.max()):.4g}")
            return worst
    return worst


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    failures, report = [], {}
    try:
        g = torch.Generator(device=dev)
        g.manual_seed(7)
        M, K, N = 1024, 1024, 2560
        X = torch.randn(M, K, generator=g, device=dev).bfloat16()
        W = (torch.randn(K, N, generator=g, device=dev) / K ** 0.5).bfloat16()
        b = (torch.rand(N, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
        Xc, Wc, bc = cpu(X), cpu(W), cpu(b)
        modules = []
        col = ColumnParallelLinear(W, b, "silu", gather_output=True)
        got = col(X)
        torch.cuda.synchronize()
        report["column"] = compare(
            "column-parallel", got,
            lambda r0, r1: oracle.fused_linear_f64(Xc[r0:r1], Wc, bc, "silu"), M, failures)

        H = 4096
        W1 = (torch.randn(K, H, generator=g, device=dev) / K ** 0.5).bfloat16()
        b1 = (torch.rand(H, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
        W2 = (torch.randn(H, K, generator=g, device=dev) / H ** 0.5).bfloat16()
        b2 = (torch.rand(K, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
        W1c, b1c, W2c, b2c = cpu(W1), cpu(b1), cpu(W2), cpu(b2)
        cache = {}

        def mlp_ref(Xh):
            def rows(r0, r1):
                key = (id(Xh), r0, r1)
                if key not in cache:
                    cache[key] = oracle.mlp_residual_f64(Xh[r0:r1], W1c, b1c, W2c, b2c, "gelu")
                return cache[key]
            return rows

        ref_rows = mlp_ref(Xc)
        for mode, chunks, first, nvls in (("nccl", 1, None, None), ("nccl", 4, None, None),
                                          ("fused", 1, None, False), ("fused", 4, None, False),
                                          ("fused", 4, 2, False), ("fused", 3, 1, False),
                                          ("fused", 1, None, True), ("fused", 4, None, True),
                                          ("fused", 4, 2, True), ("fused", 3, 1, True)):
            mlp = ParallelMLP(W1, b1, W2, b2, "gelu", chunks=chunks, mode=mode,
                              first_chunks=first, nvls=nvls)
            modules.append(mlp)
            outs = []
            for rep in range(3):  # the fused mode reuses its buffers and flips slab halves
                outs.append(mlp(X))
            torch.cuda.synchronize()
            if mlp.last_path != mode:
                failures.append(f"MLP {mode}: ran the {mlp.last_path} path")
            tag = f"{mode}{'_mc' if mlp.last_multicast else ''}"
            if nvls and mode == "fused":
                report["multicast_available"] = bool(mlp.last_multicast)
            for rep, out in enumerate(outs):
                report[f"mlp_{tag}_c{chunks}_f{first}_{rep}"] = compare(
                    f"MLP ({tag}, chunks={chunks}, first={first}, call {rep})", out, ref_rows,
                    M, failures)

        # Output ownership: a later call with other inputs leaves Y1 intact.
        mlp = ParallelMLP(W1, b1, W2, b2, "gelu", mode="fused")
        modules.append(mlp)
        X2 = torch.randn(M, K, generator=g, device=dev).bfloat16()
        Y1 = mlp(X)
        Y1_copy = Y1.clone()
        Y2 = mlp(X2)
        torch.cuda.synchronize()
        if Y1.data_ptr() == Y2.data_ptr() or not torch.equal(Y1, Y1_copy):
            failures.append("MLP fused: a second call overwrote the first call's output")
        report["mlp_second_input"] = compare("MLP fused, second input", Y2, mlp_ref(cpu(X2)), M,
                                             failures)

        # Rows the overlapped reduction cannot split evenly over the ranks.
        m_odd = world + 1 if world > 1 else 3
        Xo = X[:m_odd].contiguous()
        mlp = ParallelMLP(W1, b1, W2, b2, "gelu", mode="fused")
        out = mlp(Xo)
        torch.cuda.synchronize()
        if world > 1 and mlp.last_path != "nccl":
            failures.append(f"MLP with M={m_odd}: expected the NCCL fallback")
        report["mlp_odd_rows"] = compare(f"MLP M={m_odd}", out, mlp_ref(cpu(Xo)), m_odd,
                                         failures, blocks=[(0, m_odd)])

        Wg = (torch.randn(K, H, generator=g, device=dev) / K ** 0.5).bfloat16()
        Wu = (torch.randn(K, H, generator=g, device=dev) / K ** 0.5).bfloat16()
        bg = (torch.rand(H, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
        bu = (torch.rand(H, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
        Wgc, Wuc, bgc, buc = cpu(Wg), cpu(Wu), cpu(bg), cpu(bu)
        for mode, nvls in (("nccl", None), ("fused", False), ("fused", True)):
            ffn = ParallelGatedFFN(Wg, bg, Wu, bu, W2, b2, "silu", mode=mode, nvls=nvls)
            modules.append(ffn)
            outs = [ffn(X) for _ in range(2)]
            torch.cuda.synchronize()
            for rep, out in enumerate(outs):
                tag = f"{mode}{'_mc' if ffn.last_multicast else ''}"
                report[f"gated_{tag}_{rep}"] = compare(
                    f"gated FFN ({tag}, call {rep})", out,
                    lambda r0, r1: oracle.gated_ffn_f64(Xc[r0:r1], Wgc, bgc, Wuc, buc, W2c, b2c,
                                                        "silu"),
                    M, failures)
        status = _native.device_status(torch.cuda.current_stream(dev).cuda_stream)
        if status:
            failures.append(f"device status {status}")
        # Collective release of the peer-mapped buffers: no rank unmaps memory
        # (multicast-bound or not) while a peer's kernels may still reach it.
        for m in modules:
            m.release()
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    for f in failures:
        print(f"rank {rank}/{world}: {f}", flush=True)
    if rank == 0:
        print("max |err| vs fp64 oracle: " +
              ", ".join(f"{k}={v:.3g}" for k, v in report.items()), flush=True)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
