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
    - ``mode="fused"`` (GPUs, default): the rows are cut into chunks; each
      chunk's two GEMMs run in turn, the second writing its partial into a
      peer-mapped (symmetric-memory) buffer, and the following GEMM launches
      carry that chunk's reduce-scatter and all-gather over NVLink (peer
      loads, rank order, b2 and X added once) in their spare warps, so the
      reduction of one chunk runs on the same SMs while the next chunk's
      GEMMs compute — one stream, no NCCL on the path; the output is a
      buffer the caller owns;
    - ``mode="nccl"``: b2 and X are fused into rank 0's second launch and
      Y is summed with NCCL all-reduce (in M-chunks issued asynchronously
      when ``chunks > 1``).  This mode also runs on CPU ranks (gloo), and
      takes the shapes the fused mode cannot (M not a multiple of the world
      size — e.g. decode rows — N not a multiple of 8, fp32).
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


MAX_ROW_CHUNKS = 64  # chunk indices dx_row_reduce keeps flags for


def row_chunks(M: int, world: int, chunks: int) -> list[tuple[int, int]]:
    """(first row, rows) of the row chunks of the overlapped reduction: up to
    `chunks` near-equal chunks whose starts and sizes are multiples of
    32 * world when M allows (so every rank's slab of a chunk is a whole
    number of 32-row groups), else of world."""
    if world <= 0 or M % world:
        raise ValueError(f"M ({M}) must be a multiple of the world size ({world})")
    unit = world * 32 if M % (world * 32) == 0 else world
    units = M // unit
    n = max(1, min(int(chunks), units, MAX_ROW_CHUNKS))
    edges = [(i * units // n) * unit for i in range(n + 1)]
    return [(a, b - a) for a, b in zip(edges, edges[1:]) if b > a]


def first_groups(n_chunks: int, groups: int | None) -> list[tuple[int, int]]:
    """[start, end) chunk-index ranges that one launch of the first GEMM
    covers: `groups` near-equal runs of consecutive chunks (None: one per
    chunk)."""
    g = n_chunks if groups is None else max(1, min(int(groups), n_chunks))
    edges = [i * n_chunks // g for i in range(g + 1)]
    return [(a, b) for a, b in zip(edges, edges[1:]) if b > a]


def row_schedule(n_chunks: int, groups: list[tuple[int, int]]) -> list[tuple]:
    """Launch order of one overlapped step, in stream order:

    * ``("first", c0, c1, job)`` — the first GEMM for the rows of chunks
      [c0, c1);
    * ``("second", c, job)`` — chunk c's second GEMM (its partial);
    * ``("reduce", job)`` — a reduction launch of its own (only at the end).

    ``job = (a, b)`` names the chunk whose reduce-scatter (phase A) and the
    chunk whose all-gather (phase B) the launch carries, or None.  A chunk's
    phase A rides on the first launch after its second GEMM (the partial is
    complete by then in stream order); its phase B on a later launch than its
    phase A (so every rank's slab was announced in an earlier launch), except
    at the very end, where one launch may do both."""
    starts = dict(groups)
    plan: list[tuple] = []
    pending_a = None  # partial complete, reduce-scatter not carried yet
    gathers: list[int] = []  # reduce-scatter carried by an earlier launch

    def take():
        nonlocal pending_a
        a, pending_a = pending_a, None
        return a, (gathers.pop(0) if gathers else None)

    for c in range(n_chunks):
        if c in starts:
            job = take()
            plan.append(("first", c, starts[c], job))
            if job[0] is not None:
                gathers.append(job[0])
        job = take()
        plan.append(("second", c, job))
        if job[0] is not None:
            gathers.append(job[0])
        pending_a = c
    while pending_a is not None or gathers:
        a, pending_a = pending_a, None
        if a is not None and not gathers:
            plan.append(("reduce", (a, a)))
        else:
            plan.append(("reduce", (a, gathers.pop(0))))
            if a is not None:
                gathers.append(a)
    return plan


class _RowParallelBuffers:
    """Peer-mapped (symmetric-memory) buffers of the overlapped reduction for
    one (M, N, dtype): every rank's partial [M, N] and flag words, and either
    (NVLink multicast form) a peer-written output [M, N] bound, like the
    partials, to a multicast address, or (peer-load form) a slab buffer
    [2 * M / world, N].  The multicast form is used when `nvls` allows it
    and every rank's buffers have multicast addresses."""

    def __init__(self, M: int, N: int, dtype, device, group, nvls: bool | None):
        import os

        import torch.distributed._symmetric_memory as symm_mem

        from .linear import row_flag_words
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        pg = group if group is not None else dist.group.WORLD
        self.key = (M, N, dtype)
        self.part = symm_mem.empty(M, N, dtype=dtype, device=device)
        self.flags = symm_mem.empty(row_flag_words(), dtype=torch.int32, device=device)
        self.flags.zero_()
        torch.cuda.current_stream(device).synchronize()
        self.handles = [symm_mem.rendezvous(t, pg) for t in (self.part, self.flags)]
        self.part_ptrs = self._peer_ptrs(self.handles[0], self.part, rank)
        self.flag_ptrs = self._peer_ptrs(self.handles[1], self.flags, rank)
        self.mc_part = self.mc_out = 0
        self.out_sym = None
        self.slab_ptrs = None
        if nvls is None:
            # Multicast halves the NVLink bytes per GPU but only pays with
            # several peers (2 ranks: 1.78 ms against 1.735 with peer loads;
            # 8 ranks: 0.832 ms against 1.043).
            nvls = world > 2 and os.environ.get("DX_ROW_NVLS", "1") != "0"
        if nvls:
            self.out_sym = symm_mem.empty(M, N, dtype=dtype, device=device)
            h_out = symm_mem.rendezvous(self.out_sym, pg)
            self.handles.append(h_out)
            try:
                mc_p = self._mc_ptr(self.handles[0], self.part, rank)
                mc_o = self._mc_ptr(h_out, self.out_sym, rank)
            except RuntimeError:  # this allocation has no multicast mapping
                mc_p = mc_o = 0
            have = torch.tensor([1 if (mc_p and mc_o) else 0], device=device)
            dist.all_reduce(have, op=dist.ReduceOp.MIN, group=group)
            if int(have.item()):
                self.mc_part, self.mc_out = mc_p, mc_o
        if not self.mc_part:
            self.slab = symm_mem.empty(2 * M // world, N, dtype=dtype, device=device)
            h_slab = symm_mem.rendezvous(self.slab, pg)
            self.handles.append(h_slab)
            self.slab_ptrs = self._peer_ptrs(h_slab, self.slab, rank)
        # Every rank's flags are zero before any peer stamps them.
        dist.barrier(group=group)
        self.epoch = 0

    @property
    def multicast(self) -> bool:
        return bool(self.mc_part)

    @staticmethod
    def _peer_ptrs(handle, t: torch.Tensor, rank: int) -> list[int]:
        off = t.data_ptr() - int(handle.buffer_ptrs[rank])
        return [int(p) + off for p in handle.buffer_ptrs]

    @staticmethod
    def _mc_ptr(handle, t: torch.Tensor, rank: int) -> int:
        base = int(getattr(handle, "multicast_ptr", 0) or 0)
        return base + (t.data_ptr() - int(handle.buffer_ptrs[rank])) if base else 0


class _RowParallelOutput:
    """The row-parallel second GEMM and its reduction, shared by the FFN
    classes: Y = sum_r H_r W2_r + b2 (+ R), W2_r this rank's row shard.

    ``mode="fused"`` (the default on GPUs with world > 1): the engine's
    overlapped reduction.  The rows are cut into ``chunks`` chunks; each
    chunk's first GEMM (grouped into ``first_chunks`` launches) and second
    GEMM run in turn on the caller's stream, the second writing its partial
    into a peer-mapped buffer.  The next launch carries that chunk's
    reduce-scatter over NVLink (peer loads, rank order, b2 and R added once)
    and a later one its all-gather: the GEMM kernels' spare warps run them
    while the tensor-core warps compute (row_schedule gives the order; the
    last chunk's reduction runs as a launch of its own).  The result lands in
    a buffer the caller owns (``out``, or a new tensor).  Shapes it cannot
    take (M not a multiple of the world size, N not a multiple of 8, fp32,
    world > 8) run the NCCL path instead.
    ``mode="nccl"``: the whole first GEMM, then the second in ``chunks``
    row chunks, each summed by an asynchronous NCCL all-reduce (b2 and R
    fused into rank 0's launch).  Also runs on CPU ranks (gloo)."""

    def _init_output(self, W2_shard, b2_full, group, linear_fn, chunks, mode, on_gpu,
                     first_chunks=None, nvls=None):
        self.group = group
        self.nvls = nvls
        self.world, self.rank = _group_info(group)
        self.mode = mode or ("fused" if (linear_fn is None and on_gpu and self.world > 1)
                             else "nccl")
        self._bufs = None
        self.W2 = W2_shard
        self.b2_all = b2_full.contiguous() if b2_full is not None else None
        self.b2 = self.b2_all if self.rank == 0 else None
        self.linear_fn = linear_fn or _default_linear()
        # Defaults from measurements on one 8-GPU B200 box (16384 x 4096 x 16384
        # MLP): the reduction carried by 4 chunks' GEMMs is fully hidden at 2
        # ranks (1.735 ms, NCCL 1.847); at 8 ranks the reduction alone (~0.44
        # ms at the fabric's all-to-all rate) outlasts the compute (0.41 ms)
        # and chunked GEMMs lose efficiency, so one chunk — the whole GEMMs,
        # then one reduction launch — is fastest (0.832 ms, NCCL 1.01).
        if chunks is None:
            chunks = 1 if self.mode != "fused" else (4 if self.world <= 2 else
                                                     2 if self.world <= 4 else 1)
        self.chunks = max(1, int(chunks))
        self.first_chunks = first_chunks
        # Called with (index, launch) before each launch of an overlapped step
        # (launch as row_schedule gives it): a profiling aid, e.g. to switch
        # dx_set_trace_buffer between launches.
        self.launch_hook = None
        self.last_path = None  # "fused" or "nccl": what the last call ran
        self.last_multicast = False  # the last fused call used NVLink multicast

    def _fused_ok(self, M: int, N: int, dtype) -> bool:
        return (self.mode == "fused" and 1 < self.world <= 8 and M % self.world == 0
                and N % 8 == 0 and dtype in (torch.float16, torch.bfloat16))

    def _run(self, first, M: int, H: torch.Tensor, R: torch.Tensor | None,
             out: torch.Tensor | None) -> torch.Tensor:
        """Y for rows [0, M): `first(r0, r1)` fills H[r0:r1] (the chain's
        first GEMM), then the row-parallel second GEMM and its reduction."""
        N = self.W2.shape[1]
        if self._fused_ok(M, N, H.dtype):
            Y = self._run_overlapped(first, M, H, R, out)
            self.last_path = "fused"
            self.last_multicast = self._bufs.multicast
            return Y
        self.last_path = "nccl"
        first(0, M)
        return self._row_parallel_nccl(H, R, out)

    def release(self) -> None:
        """Drop the peer-mapped buffers.  Collective: every rank calls it,
        with no step of this module in flight on any rank (it synchronises
        the device and the group first), so no rank unmaps memory that a
        peer's multicast or peer accesses may still reach."""
        if self._bufs is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            self._bufs = None
            dist.barrier(group=self.group)

    def _row_parallel_nccl(self, H: torch.Tensor, R: torch.Tensor | None,
                           out: torch.Tensor | None) -> torch.Tensor:
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

    def _run_overlapped(self, first, M: int, H: torch.Tensor, R: torch.Tensor | None,
                        out: torch.Tensor | None) -> torch.Tensor:
        from .linear import fused_linear, row_job, row_reduce
        N = self.W2.shape[1]
        dev = H.device
        key = (M, N, H.dtype)
        if self._bufs is None or self._bufs.key != key:
            self._bufs = None
            self._bufs = _RowParallelBuffers(M, N, H.dtype, dev, self.group, self.nvls)
        bufs = self._bufs
        Y = out if out is not None else torch.empty((M, N), dtype=H.dtype, device=dev)
        chunks = row_chunks(M, self.world, self.chunks)
        plan = row_schedule(len(chunks), first_groups(len(chunks), self.first_chunks))
        bufs.epoch += 1

        def job(ab):
            a, b = ab
            if a is None and b is None:
                return None
            return row_job(bufs.part_ptrs, bufs.slab_ptrs, bufs.flag_ptrs, self.rank, M, N, N,
                           (chunks[a][0], chunks[a][1], a) if a is not None else None,
                           (chunks[b][0], chunks[b][1], b) if b is not None else None,
                           self.b2_all, R, Y, bufs.epoch, H.dtype, bufs.mc_part, bufs.mc_out,
                           bufs.out_sym)

        stream = torch.cuda.current_stream(dev).cuda_stream
        for i, launch in enumerate(plan):
            if self.launch_hook is not None:
                self.launch_hook(i, launch)
            if launch[0] == "first":
                _, c0, c1, ab = launch
                first(chunks[c0][0], chunks[c1 - 1][0] + chunks[c1 - 1][1], job(ab))
            elif launch[0] == "second":
                _, c, ab = launch
                r0, rn = chunks[c]
                fused_linear(H[r0:r0 + rn], self.W2, None, None, out=bufs.part[r0:r0 + rn],
                             row_job=job(ab))
            else:
                row_reduce(job(launch[1]), stream)
        return Y


class ParallelMLP(_RowParallelOutput):
    """Y = act(X W1 + b1) W2 + b2 + X with W1 column- and W2 row-sharded."""

    def __init__(self, W1_full, b1_full, W2_full, b2_full, activation="gelu", group=None,
                 linear_fn=None, chunks: int | None = None, align: int = 64,
                 mode: str | None = None, first_chunks: int | None = None,
                 nvls: bool | None = None):
        world, rank = _group_info(group)
        hidden = W1_full.shape[1]
        if W2_full.shape[0] != hidden:
            raise ValueError("W1 columns and W2 rows must match")
        self.h0, self.h1 = shard_bounds(hidden, world, rank, align)
        self.W1 = W1_full[:, self.h0:self.h1].contiguous()
        self.b1 = b1_full[self.h0:self.h1].contiguous() if b1_full is not None else None
        self.activation = activation
        self._init_output(W2_full[self.h0:self.h1, :].contiguous(), b2_full, group, linear_fn,
                          chunks, mode, on_gpu=W1_full.is_cuda, first_chunks=first_chunks,
                          nvls=nvls)

    @classmethod
    def from_shards(cls, W1_shard, b1_shard, W2_shard, b2_full, activation="gelu", group=None,
                    linear_fn=None, chunks: int | None = None, mode: str | None = None,
                    first_chunks: int | None = None, nvls: bool | None = None):
        self = cls.__new__(cls)
        self.W1, self.b1 = W1_shard, b1_shard
        self.activation = activation
        self._init_output(W2_shard, b2_full, group, linear_fn, chunks, mode,
                          on_gpu=W1_shard.is_cuda, first_chunks=first_chunks, nvls=nvls)
        return self

    def __call__(self, X: torch.Tensor, hidden: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        M = X.shape[0]
        H = hidden if hidden is not None else torch.empty(
            (M, self.W1.shape[1]), dtype=X.dtype, device=X.device)

        def first(r0: int, r1: int, job=None) -> None:
            kw = {"row_job": job} if job is not None else {}
            self.linear_fn(X[r0:r1], self.W1, self.b1, self.activation, out=H[r0:r1], **kw)

        return self._run(first, M, H, X, out)


class ParallelGatedFFN(_RowParallelOutput):
    """Y = (act(X Wg + bg) * (X Wu + bu)) Wo + bo with Wg, Wu column- and Wo
    row-sharded on the same hidden slice (the ``ffn_gated`` chain)."""

    def __init__(self, Wg_full, bg_full, Wu_full, bu_full, Wo_full, bo_full, activation="silu",
                 group=None, gated_fn=None, linear_fn=None, chunks: int | None = None,
                 align: int = 64, mode: str | None = None, first_chunks: int | None = None,
                 nvls: bool | None = None):
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
                          linear_fn, chunks, mode, first_chunks, nvls)
        self.h0, self.h1 = h0, h1

    @classmethod
    def from_shards(cls, Wg_shard, bg_shard, Wu_shard, bu_shard, Wo_shard, bo_full,
                    activation="silu", group=None, gated_fn=None, linear_fn=None,
                    chunks: int | None = None, mode: str | None = None,
                    first_chunks: int | None = None, nvls: bool | None = None):
        self = cls.__new__(cls)
        self._init_shards(Wg_shard, bg_shard, Wu_shard, bu_shard, Wo_shard, bo_full, activation,
                          group, gated_fn, linear_fn, chunks, mode, first_chunks, nvls)
        return self

    def _init_shards(self, Wg, bg, Wu, bu, Wo, bo_full, activation, group, gated_fn, linear_fn,
                     chunks, mode, first_chunks=None, nvls=None):
        self.Wg, self.bg, self.Wu, self.bu = Wg, bg, Wu, bu
        self.activation = activation
        self.gated_fn = gated_fn or _default_gated()
        self._init_output(Wo, bo_full, group, linear_fn, chunks, mode,
                          on_gpu=Wg.is_cuda and gated_fn is None, first_chunks=first_chunks,
                          nvls=nvls)

    def __call__(self, X: torch.Tensor, hidden: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        M = X.shape[0]
        H = hidden if hidden is not None else torch.empty(
            (M, self.Wg.shape[1]), dtype=X.dtype, device=X.device)

        def first(r0: int, r1: int, job=None) -> None:
            kw = {"row_job": job} if job is not None else {}
            self.gated_fn(X[r0:r1], self.Wg, self.Wu, self.bg, self.bu, self.activation,
                          out=H[r0:r1], **kw)

        return self._run(first, M, H, None, out)
