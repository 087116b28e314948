"""Megatron-style partitioning of the fused linear over ranks (one per GPU).

The reference runs on one GPU only.  Large problems are split here the
standard way, one process per GPU over ``torch.distributed`` (NCCL on GPUs):

* ``ColumnParallelLinear`` — a single fused layer Y = act(X W + b): rank r
  owns the column slice W[:, n_r0:n_r1] and bias[n_r0:n_r1] and produces
  Y[:, n_r0:n_r1].  No data-path collective (``gather_output=True`` adds an
  all-gather for callers that need the full Y on every rank).
* ``ParallelMLP`` — the two-GEMM chain Y = act(X W1 + b1) W2 + b2 + X:
  W1 column-sharded, W2 row-sharded with the same hidden slice, so
  H_r = act(X W1_r + b1_r) stays local and Y = sum_r H_r W2_r needs one
  all-reduce.  Two implementations:
    - ``mode="fused"`` (GPUs, default): the second GEMM writes its partial
      into a peer-mapped (symmetric-memory) buffer; after a device barrier
      each rank reads its row slab from every rank's partial over NVLink,
      sums in rank order, adds b2 and X once and writes the finished rows
      into every rank's output (one engine kernel, dx_reduce_broadcast) —
      no NCCL on the path;
    - ``mode="nccl"``: b2 and X are fused into rank 0's second launch and
      Y is summed with NCCL all-reduce (in M-chunks issued asynchronously
      when ``chunks > 1``).  This mode also runs on CPU ranks (gloo).
* ``ParallelGatedFFN`` — the ``ffn_gated`` chain (fusion.py:44-46)
  Y = (act(X Wg + bg) * (X Wu + bu)) Wo + bo: Wg and Wu column-sharded on
  the same hidden slice (one gated dual-GEMM launch per rank), Wo
  row-sharded, and the same two reductions (no residual).

Shard boundaries are multiples of ``align`` elements (default 64) so every
slice of a row-major matrix starts on a 128-byte boundary and stays
addressable by TMA.  The compute function is injectable (``linear_fn``,
signature of ``linear.fused_linear``) so the partitioning logic can be run
on CPU ranks in tests; by default it is the B200 engine.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(n: int, world: int, rank: int, align: int = 64) -> tuple[int, int]:
    """[start, end) of rank's slice of n items; boundaries are multiples of
    `align` (except the final end), slices as even as that allows."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    units = (n + align - 1) // align
    base, extra = divmod(units, world)
    start_u = rank * base + min(rank, extra)
    end_u = start_u + base + (1 if rank < extra else 0)
    return min(start_u * align, n), min(end_u * align, n)


def _default_linear():
    from .linear import fused_linear
    return fused_linear


def _default_gated():
    from .linear import fused_gated_linear
    return fused_gated_linear


def _group_info(group):
    return dist.get_world_size(group), dist.get_rank(group)


class ColumnParallelLinear:
    """Y[:, slice_r] = act(X @ W[:, slice_r] + b[slice_r]) on every rank."""

    def __init__(self, W_full: torch.Tensor, bias_full: torch.Tensor | None, activation=None,
                 group=None, gather_output: bool = False, linear_fn=None, align: int = 64):
        world, rank = _group_info(group)
        self.group, self.world, self.rank = group, world, rank
        self.n_total = W_full.shape[1]
        self.align = align
        self.n0, self.n1 = shard_bounds(self.n_total, world, rank, align)
        self.W = W_full[:, self.n0:self.n1].contiguous()
        self.bias = bias_full[self.n0:self.n1].contiguous() if bias_full is not None else None
        self.activation = activation
        self.gather_output = gather_output
        self.linear_fn = linear_fn or _default_linear()

    @classmethod
    def from_shard(cls, W_shard, bias_shard, n_total: int, n0: int, activation=None, group=None,
                   gather_output: bool = False, linear_fn=None):
        """Build from a shard the caller already holds (no full matrix)."""
        self = cls.__new__(cls)
        self.group = group
        self.world, self.rank = _group_info(group)
        self.n_total, self.n0, self.n1 = n_total, n0, n0 + W_shard.shape[1]
        self.align = 64
        self.W, self.bias = W_shard, bias_shard
        self.activation, self.gather_output = activation, gather_output
        self.linear_fn = linear_fn or _default_linear()
        return self

    def __call__(self, X: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        Y = self.linear_fn(X, self.W, self.bias, self.activation, out=out)
        if not self.gather_output:
            return Y
        bounds = [shard_bounds(self.n_total, self.world, r, self.align) for r in range(self.world)]
        sizes = [e - s for s, e in bounds]
        # Shards may differ in width; gather equal-size padded blocks.
        width = max(sizes)
        buf = torch.zeros((X.shape[0], width), dtype=Y.dtype, device=Y.device)
        buf[:, :Y.shape[1]] = Y
        parts = [torch.empty_like(buf) for _ in range(self.world)]
        dist.all_gather(parts, buf, group=self.group)
        return torch.cat([p[:, :sz] for p, sz in zip(parts, sizes)], dim=1)


class _RowParallelBuffers:
    """Symmetric (peer-mapped) partial and output buffers of one shape."""

    def __init__(self, M: int, N: int, dtype, device, group):
        import torch.distributed._symmetric_memory as symm_mem
        world = dist.get_world_size(group)
        if M % world:
            raise ValueError(f"fused row-parallel needs M ({M}) divisible by world ({world})")
        self.key = (M, N, dtype)
        self.rows_per_rank = M // world
        self.part = symm_mem.empty(M, N, dtype=dtype, device=device)
        self.out = symm_mem.empty(M, N, dtype=dtype, device=device)
        pg = group if group is not None else dist.group.WORLD
        self.h_part = symm_mem.rendezvous(self.part, pg)
        self.h_out = symm_mem.rendezvous(self.out, pg)
        self.part_ptrs = list(self.h_part.buffer_ptrs)
        self.out_ptrs = list(self.h_out.buffer_ptrs)


class _RowParallelOutput:
    """The row-parallel second GEMM and its reduction, shared by the FFN
    classes: Y = sum_r H_r W2_r + b2 (+ R), W2_r this rank's row shard."""

    def _init_output(self, W2_shard, b2_full, group, linear_fn, chunks, mode, on_gpu):
        self.group = group
        self.world, self.rank = _group_info(group)
        self.mode = mode or ("fused" if (linear_fn is None and on_gpu and self.world > 1)
                             else "nccl")
        self._bufs = None
        self.W2 = W2_shard
        self.b2_all = b2_full.contiguous() if b2_full is not None else None
        self.b2 = self.b2_all if self.rank == 0 else None
        self.linear_fn = linear_fn or _default_linear()
        self.chunks = max(1, int(chunks))

    def _row_parallel(self, H: torch.Tensor, R: torch.Tensor | None,
                      out: torch.Tensor | None) -> torch.Tensor:
        if self.mode == "fused":
            return self._row_parallel_fused(H, R, out)
        M = H.shape[0]
        Y = out if out is not None else torch.empty((M, self.W2.shape[1]), dtype=H.dtype,
                                                    device=H.device)
        residual_rank = self.rank == 0
        handles = []
        step = (M + self.chunks - 1) // self.chunks
        for m0 in range(0, M, step):
            m1 = min(M, m0 + step)
            self.linear_fn(H[m0:m1], self.W2, self.b2, None,
                           residual=R[m0:m1] if (residual_rank and R is not None) else None,
                           out=Y[m0:m1])
            if self.world > 1:
                handles.append(dist.all_reduce(Y[m0:m1], op=dist.ReduceOp.SUM, group=self.group,
                                               async_op=True))
        for h in handles:
            h.wait()
        return Y

    def _row_parallel_fused(self, H: torch.Tensor, R: torch.Tensor | None,
                            out: torch.Tensor | None) -> torch.Tensor:
        """Y = sum_r H_r W2_r + b2 (+ R): local partial, then reduce-broadcast."""
        from .linear import fused_linear, reduce_broadcast
        M, N = H.shape[0], self.W2.shape[1]
        key = (M, N, H.dtype)
        if self._bufs is None or self._bufs.key != key:
            self._bufs = _RowParallelBuffers(M, N, H.dtype, H.device, self.group)
        bufs = self._bufs
        rpr = bufs.rows_per_rank
        fused_linear(H, self.W2, None, None, out=bufs.part)
        bufs.h_part.barrier(channel=0)  # every rank's partial is complete
        reduce_broadcast(bufs.part, bufs.part_ptrs, self.rank, rpr, self.b2_all, R,
                         bufs.out_ptrs, N)
        # Every rank's rows have landed, and no rank still reads a partial
        # that the next call will overwrite.
        bufs.h_out.barrier(channel=1)
        if out is None:
            return bufs.out
        out.copy_(bufs.out)
        return out


class ParallelMLP(_RowParallelOutput):
    """Y = act(X W1 + b1) W2 + b2 + X with W1 column- and W2 row-sharded."""

    def __init__(self, W1_full, b1_full, W2_full, b2_full, activation="gelu", group=None,
                 linear_fn=None, chunks: int = 1, align: int = 64, mode: str | None = None):
        world, rank = _group_info(group)
        hidden = W1_full.shape[1]
        if W2_full.shape[0] != hidden:
            raise ValueError("W1 columns and W2 rows must match")
        self.h0, self.h1 = shard_bounds(hidden, world, rank, align)
        self.W1 = W1_full[:, self.h0:self.h1].contiguous()
        self.b1 = b1_full[self.h0:self.h1].contiguous() if b1_full is not None else None
        self.activation = activation
        self._init_output(W2_full[self.h0:self.h1, :].contiguous(), b2_full, group, linear_fn,
                          chunks, mode, on_gpu=W1_full.is_cuda)

    @classmethod
    def from_shards(cls, W1_shard, b1_shard, W2_shard, b2_full, activation="gelu", group=None,
                    linear_fn=None, chunks: int = 1, mode: str | None = None):
        self = cls.__new__(cls)
        self.W1, self.b1 = W1_shard, b1_shard
        self.activation = activation
        self._init_output(W2_shard, b2_full, group, linear_fn, chunks, mode,
                          on_gpu=W1_shard.is_cuda)
        return self

    def __call__(self, X: torch.Tensor, hidden: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        H = self.linear_fn(X, self.W1, self.b1, self.activation, out=hidden)
        return self._row_parallel(H, X, out)


class ParallelGatedFFN(_RowParallelOutput):
    """Y = (act(X Wg + bg) * (X Wu + bu)) Wo + bo with Wg, Wu column- and Wo
    row-sharded on the same hidden slice (the ``ffn_gated`` chain)."""

    def __init__(self, Wg_full, bg_full, Wu_full, bu_full, Wo_full, bo_full, activation="silu",
                 group=None, gated_fn=None, linear_fn=None, chunks: int = 1, align: int = 64,
                 mode: str | None = None):
        world, rank = _group_info(group)
        hidden = Wg_full.shape[1]
        if Wu_full.shape != Wg_full.shape or Wo_full.shape[0] != hidden:
            raise ValueError("Wg and Wu must match, and Wo must take their column count as rows")
        h0, h1 = shard_bounds(hidden, world, rank, align)
        sl = slice(h0, h1)
        self._init_shards(Wg_full[:, sl].contiguous(),
                          bg_full[sl].contiguous() if bg_full is not None else None,
                          Wu_full[:, sl].contiguous(),
                          bu_full[sl].contiguous() if bu_full is not None else None,
                          Wo_full[sl, :].contiguous(), bo_full, activation, group, gated_fn,
                          linear_fn, chunks, mode)
        self.h0, self.h1 = h0, h1

    @classmethod
    def from_shards(cls, Wg_shard, bg_shard, Wu_shard, bu_shard, Wo_shard, bo_full,
                    activation="silu", group=None, gated_fn=None, linear_fn=None,
                    chunks: int = 1, mode: str | None = None):
        self = cls.__new__(cls)
        self._init_shards(Wg_shard, bg_shard, Wu_shard, bu_shard, Wo_shard, bo_full, activation,
                          group, gated_fn, linear_fn, chunks, mode)
        return self

    def _init_shards(self, Wg, bg, Wu, bu, Wo, bo_full, activation, group, gated_fn, linear_fn,
                     chunks, mode):
        self.Wg, self.bg, self.Wu, self.bu = Wg, bg, Wu, bu
        self.activation = activation
        self.gated_fn = gated_fn or _default_gated()
        self._init_output(Wo, bo_full, group, linear_fn, chunks, mode,
                          on_gpu=Wg.is_cuda and gated_fn is None)

    def __call__(self, X: torch.Tensor, hidden: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        H = self.gated_fn(X, self.Wg, self.Wu, self.bg, self.bu, self.activation, out=hidden)
        return self._row_parallel(H, None, out)
