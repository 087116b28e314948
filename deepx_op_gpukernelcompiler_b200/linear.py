"""PyTorch-facing wrapper of the fused linear C ABI.

``fused_linear(X, W, bias, activation, residual)`` computes
``act(X @ W + bias) + residual`` on the tensors' CUDA device, on the current
stream, through ``dx_fused_linear`` (include/deepx_fused.h).  PyTorch only
provides device memory and the stream; the arithmetic runs in the sm_100a
kernels of ``csrc/``.  Inputs must be CUDA tensors — there is no CPU path.

Activation names follow the reference: ``relu``, ``gelu`` (tanh
approximation, as ``ACTIVATION_PT['gelu']`` in fusion.py:89), ``silu`` and
``swish`` (= silu, fusion.py:91), plus the explicit ``gelu_tanh`` /
``gelu_erf`` (the erf form is what kernel_triton.py:61 and
kernel_tilelang.py:17 compute).
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _native as nat

ACTIVATION_CODES = {
    None: nat.DX_ACT_NONE,
    "none": nat.DX_ACT_NONE,
    "relu": nat.DX_ACT_RELU,
    "gelu": nat.DX_ACT_GELU_TANH,
    "gelu_tanh": nat.DX_ACT_GELU_TANH,
    "gelu_erf": nat.DX_ACT_GELU_ERF,
    "silu": nat.DX_ACT_SILU,
    "swish": nat.DX_ACT_SILU,
}

DTYPE_CODES = {
    torch.float32: nat.DX_DTYPE_F32,
    torch.float16: nat.DX_DTYPE_F16,
    torch.bfloat16: nat.DX_DTYPE_BF16,
}

# Zero-filled workspaces, one per (device, stream): the decode kernel leaves
# its tickets at zero after every call, so a buffer is reused as is.  A
# workspace is never shared by two streams, so concurrent calls cannot race.
_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def activation_code(activation) -> int:
    try:
        return ACTIVATION_CODES[activation]
    except KeyError:
        raise ValueError(f"unsupported activation {activation!r}; expected one of "
                         f"{sorted(k for k in ACTIVATION_CODES if k)}") from None


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    key = (device.index, stream)
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _workspaces[key] = buf
        return buf


def reset_workspaces() -> None:
    """Drop cached workspaces (after a device timeout left tickets set)."""
    with _ws_lock:
        _workspaces.clear()


def _check_matrix(name: str, t: torch.Tensor, rows: int | None, cols: int | None) -> None:
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D, got shape {tuple(t.shape)}")
    if rows is not None and t.shape[0] != rows:
        raise ValueError(f"{name} has {t.shape[0]} rows, expected {rows}")
    if cols is not None and t.shape[1] != cols:
        raise ValueError(f"{name} has {t.shape[1]} columns, expected {cols}")
    if t.shape[1] > 1 and t.stride(1) != 1:
        raise ValueError(f"{name} must have unit stride along its last dimension")
    if t.shape[0] > 1 and t.stride(0) < t.shape[1]:
        raise ValueError(f"{name} rows overlap (stride {t.stride(0)} < {t.shape[1]})")


def _ld(t: torch.Tensor) -> int:
    return max(t.stride(0), t.shape[1], 1) if t.shape[0] > 1 else max(t.shape[1], 1)


def fused_linear(X: torch.Tensor, W: torch.Tensor, bias: torch.Tensor | None = None,
                 activation=None, residual: torch.Tensor | None = None,
                 out: torch.Tensor | None = None, kernel: str = "auto",
                 row_job=None) -> torch.Tensor:
    """Y = act(X @ W + bias) + residual, one fused launch on X's device.

    `row_job` (a ``_native.RowReduceJob``, see row_job()) is a chunk of a
    row-parallel reduction that the launch carries: its spare warps run it
    while the GEMM computes (dx_fused_linear_rowjob)."""
    act = activation_code(activation)
    if kernel not in nat.KERNEL_NAMES:
        raise ValueError(f"unknown kernel {kernel!r}; expected one of {list(nat.KERNEL_NAMES)}")
    if not isinstance(X, torch.Tensor) or not isinstance(W, torch.Tensor):
        raise TypeError("X and W must be torch tensors")
    if X.device.type != "cuda":
        raise ValueError("fused_linear runs on CUDA tensors only (the engine has no CPU path)")
    if X.dtype not in DTYPE_CODES:
        raise ValueError(f"unsupported dtype {X.dtype}; expected float32, float16 or bfloat16")
    _check_matrix("X", X, None, None)
    M, K = X.shape
    _check_matrix("W", W, K, None)
    N = W.shape[1]
    tensors = {"W": W}
    if bias is not None:
        if bias.dim() != 1 or bias.shape[0] != N:
            raise ValueError(f"bias must have shape ({N},), got {tuple(bias.shape)}")
        if not bias.is_contiguous():
            raise ValueError("bias must be contiguous")
        tensors["bias"] = bias
    if residual is not None:
        _check_matrix("residual", residual, M, N)
        tensors["residual"] = residual
    if out is None:
        out = torch.empty((M, N), dtype=X.dtype, device=X.device)
    else:
        _check_matrix("out", out, M, N)
        tensors["out"] = out
    for name, t in tensors.items():
        if t.dtype != X.dtype:
            raise ValueError(f"{name} dtype {t.dtype} differs from X dtype {X.dtype}")
        if t.device != X.device:
            raise ValueError(f"{name} is on {t.device}, X is on {X.device}")

    lib = nat.load()
    dtype = DTYPE_CODES[X.dtype]
    kcode = nat.KERNEL_NAMES[kernel]
    with torch.cuda.device(X.device):
        stream = torch.cuda.current_stream(X.device).cuda_stream
        ws_bytes = lib.dx_fused_linear_workspace_size(M, N, K, dtype, kcode)
        ws = _workspace(X.device, stream, ws_bytes)
        args = (X.data_ptr(), W.data_ptr(),
                bias.data_ptr() if bias is not None else None,
                residual.data_ptr() if residual is not None else None,
                out.data_ptr(), M, N, K, _ld(X), _ld(W),
                _ld(residual) if residual is not None else 0, _ld(out),
                dtype, act, kcode,
                ws.data_ptr() if ws is not None else None,
                ws.numel() if ws is not None else 0)
        if row_job is None:
            rc = lib.dx_fused_linear_ex(*args, stream)
        else:
            rc = lib.dx_fused_linear_rowjob(*args, ctypes.byref(row_job), stream)
    nat.check("dx_fused_linear", rc)
    return out


def fused_gated_linear(X: torch.Tensor, Wg: torch.Tensor, Wu: torch.Tensor,
                       bias_g: torch.Tensor | None = None, bias_u: torch.Tensor | None = None,
                       activation="silu", out: torch.Tensor | None = None,
                       kernel: str = "auto", row_job=None) -> torch.Tensor:
    """Y = act(X @ Wg + bias_g) * (X @ Wu + bias_u) in one launch
    (dx_fused_gated_linear): the first two GEMMs of the gated FFN chain
    ``ffn_gated`` (fusion.py:44-46), X read once for both weights.
    `row_job` as for fused_linear."""
    act = activation_code(activation)
    if kernel not in nat.KERNEL_NAMES:
        raise ValueError(f"unknown kernel {kernel!r}; expected one of {list(nat.KERNEL_NAMES)}")
    if X.device.type != "cuda":
        raise ValueError("fused_gated_linear runs on CUDA tensors only (the engine has no CPU path)")
    if X.dtype not in DTYPE_CODES:
        raise ValueError(f"unsupported dtype {X.dtype}; expected float32, float16 or bfloat16")
    _check_matrix("X", X, None, None)
    M, K = X.shape
    _check_matrix("Wg", Wg, K, None)
    N = Wg.shape[1]
    _check_matrix("Wu", Wu, K, N)
    tensors = {"Wg": Wg, "Wu": Wu}
    for name, b in (("bias_g", bias_g), ("bias_u", bias_u)):
        if b is not None:
            if b.dim() != 1 or b.shape[0] != N or not b.is_contiguous():
                raise ValueError(f"{name} must be a contiguous tensor of shape ({N},)")
            tensors[name] = b
    if out is None:
        out = torch.empty((M, N), dtype=X.dtype, device=X.device)
    else:
        _check_matrix("out", out, M, N)
        tensors["out"] = out
    for name, t in tensors.items():
        if t.dtype != X.dtype:
            raise ValueError(f"{name} dtype {t.dtype} differs from X dtype {X.dtype}")
        if t.device != X.device:
            raise ValueError(f"{name} is on {t.device}, X is on {X.device}")

    lib = nat.load()
    dtype = DTYPE_CODES[X.dtype]
    kcode = nat.KERNEL_NAMES[kernel]
    with torch.cuda.device(X.device):
        stream = torch.cuda.current_stream(X.device).cuda_stream
        ws = _workspace(X.device, stream,
                        lib.dx_fused_gated_linear_workspace_size(M, N, K, dtype, kcode))
        args = (X.data_ptr(), Wg.data_ptr(), Wu.data_ptr(),
                bias_g.data_ptr() if bias_g is not None else None,
                bias_u.data_ptr() if bias_u is not None else None,
                out.data_ptr(), M, N, K, _ld(X), _ld(Wg), _ld(Wu), _ld(out), dtype, act, kcode,
                ws.data_ptr() if ws is not None else None,
                ws.numel() if ws is not None else 0)
        if row_job is None:
            rc = lib.dx_fused_gated_linear(*args, stream)
        else:
            rc = lib.dx_fused_gated_linear_rowjob(*args, ctypes.byref(row_job), stream)
    nat.check("dx_fused_gated_linear", rc)
    return out


# Device buffers and side streams of fused_linear_host, per (device, calling
# stream, shape): calls on different streams never share buffers.
_host_lock = threading.Lock()
_host_states: dict[tuple, "_HostState"] = {}


class _HostState:
    def __init__(self, device: torch.device, M: int, N: int, K: int, dtype: torch.dtype):
        self.Xd = torch.empty((M, K), dtype=dtype, device=device)
        self.Wd = torch.empty((K, N), dtype=dtype, device=device)
        self.bd = torch.empty((N,), dtype=dtype, device=device)
        self.Yd = torch.empty((M, N), dtype=dtype, device=device)
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)


def release_host_buffers() -> None:
    """Free the device buffers cached by fused_linear_host."""
    with _host_lock:
        _host_states.clear()


def _block_bounds(n: int, blocks: int, align: int) -> list[tuple[int, int]]:
    units = (n + align - 1) // align
    blocks = max(1, min(blocks, units))
    out = []
    for j in range(blocks):
        u0, u1 = j * units // blocks, (j + 1) * units // blocks
        out.append((min(u0 * align, n), min(u1 * align, n)))
    return [b for b in out if b[1] > b[0]]


def _load_order(rows, cols) -> list[tuple[str, int]]:
    """Order in which X's row blocks ("r") and W's column blocks ("c") are
    copied in: row 0 and column 0 first, then whichever of the next row or
    next column block adds more computable output per element copied — the
    next row block when the loaded columns are at least as wide as the loaded
    rows are tall, else the next column block.  The loaded region grows as a
    square, so output blocks become ready early and the device-to-host copy
    of Y (the larger transfer) starts early and stays busy."""
    order = [("r", 0), ("c", 0)]
    ri, ci = 1, 1
    tall, wide = rows[0][1] - rows[0][0], cols[0][1] - cols[0][0]
    while ri < len(rows) or ci < len(cols):
        if ri < len(rows) and (ci >= len(cols) or wide >= tall):
            order.append(("r", ri))
            tall += rows[ri][1] - rows[ri][0]
            ri += 1
        else:
            order.append(("c", ci))
            wide += cols[ci][1] - cols[ci][0]
            ci += 1
    return order


def fused_linear_host(X: torch.Tensor, W: torch.Tensor, bias: torch.Tensor | None = None,
                      activation=None, out: torch.Tensor | None = None, device=None,
                      col_blocks: int | None = None, row_blocks: int | None = None,
                      kernel: str = "auto") -> torch.Tensor:
    """Y = act(X @ W + bias) for tensors in host memory, computed on `device`.

    The problem is cut into row_blocks x col_blocks output blocks (boundaries
    multiples of 256; by default up to 4 x 8 blocks of at least 2048 rows and
    1792 columns: a strided copy of rows narrower than 3.5 KB runs at half
    the PCIe rate, and smaller blocks cost more per copy and per launch than
    an earlier first output block saves — 8192x4096x14336 bf16: 6.13 ms at
    4 x 8, 6.26 ms at 2 x 4, 6.71 ms at 8 x 8).  On a copy stream, X's row
    blocks and W's column blocks go to the device in an expanding-square
    order (_load_order); each output
    block is one fused launch on the current stream as soon as its row and
    column blocks are in; on a second copy stream each finished block of Y
    returns to `out` (strided, dx_copy_2d_async) while later blocks are still
    copied in or computed.  The current stream waits for the last copy, so
    `out` is complete once it is synchronised.  Pass pinned tensors: pageable
    memory makes the copies synchronous.  W and bias are copied on every call
    (host-resident weights)."""
    if X.device.type != "cpu" or W.device.type != "cpu":
        raise ValueError("fused_linear_host takes host tensors; use fused_linear for device tensors")
    if X.dtype not in DTYPE_CODES:
        raise ValueError(f"unsupported dtype {X.dtype}; expected float32, float16 or bfloat16")
    _check_matrix("X", X, None, None)
    M, K = X.shape
    _check_matrix("W", W, K, None)
    N = W.shape[1]
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != N or not bias.is_contiguous()):
        raise ValueError(f"bias must be a contiguous tensor of shape ({N},)")
    for name, t in (("W", W), ("bias", bias), ("out", out)):
        if t is not None and (t.dtype != X.dtype or t.device.type != "cpu"):
            raise ValueError(f"{name} must be a host tensor of dtype {X.dtype}")
    if out is None:
        out = torch.empty((M, N), dtype=X.dtype, pin_memory=True)
    _check_matrix("out", out, M, N)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    caller = torch.cuda.current_stream(dev).cuda_stream
    key = (dev.index, caller, M, N, K, X.dtype)
    with _host_lock:
        st = _host_states.get(key)
        if st is None:
            st = _host_states[key] = _HostState(dev, M, N, K, X.dtype)
    lib = nat.load()
    esz = X.element_size()
    if row_blocks is None:
        row_blocks = max(1, min(4, M // 2048))
    if col_blocks is None:
        col_blocks = max(1, min(8, N // 1792))
    rows = _block_bounds(M, row_blocks, 256)
    cols = _block_bounds(N, col_blocks, 256)

    def copy2d(dst_ptr, dst_ld, src_ptr, src_ld, width, nrows, stream):
        nat.check("dx_copy_2d_async", lib.dx_copy_2d_async(
            dst_ptr, dst_ld * esz, src_ptr, src_ld * esz, width * esz, nrows, stream))

    with torch.cuda.device(dev):
        cur = torch.cuda.current_stream(dev)
        st.h2d.wait_stream(cur)  # the device buffers are free
        st.d2h.wait_stream(cur)
        h2d, d2h = st.h2d.cuda_stream, st.d2h.cuda_stream
        if bias is not None:
            copy2d(st.bd.data_ptr(), N, bias.data_ptr(), N, N, 1, h2d)
        ev_x, ev_w = {}, {}
        blocks, have_rows, have_cols = [], [], []
        for kind, i in _load_order(rows, cols):
            if kind == "r":
                m0, m1 = rows[i]
                copy2d(st.Xd.data_ptr() + m0 * K * esz, K, X.data_ptr() + m0 * _ld(X) * esz,
                       _ld(X), K, m1 - m0, h2d)
                ev_x[i] = st.h2d.record_event()
                have_rows.append(i)
                blocks += [(i, j) for j in have_cols]
            else:
                n0, n1 = cols[i]
                copy2d(st.Wd.data_ptr() + n0 * esz, N, W.data_ptr() + n0 * esz, _ld(W), n1 - n0,
                       K, h2d)
                ev_w[i] = st.h2d.record_event()
                have_cols.append(i)
                blocks += [(r, i) for r in have_rows]
        for i, j in blocks:  # in the order their inputs arrive
            (m0, m1), (n0, n1) = rows[i], cols[j]
            cur.wait_event(ev_x[i])
            cur.wait_event(ev_w[j])
            fused_linear(st.Xd[m0:m1], st.Wd[:, n0:n1],
                         st.bd[n0:n1] if bias is not None else None, activation,
                         out=st.Yd[m0:m1, n0:n1], kernel=kernel)
            st.d2h.wait_event(cur.record_event())
            copy2d(out.data_ptr() + (m0 * _ld(out) + n0) * esz, _ld(out),
                   st.Yd.data_ptr() + (m0 * N + n0) * esz, N, n1 - n0, m1 - m0, d2h)
        cur.wait_stream(st.d2h)
    return out


def selected_kernel(M: int, N: int, K: int, dtype: torch.dtype) -> str:
    """Name of the kernel variant the engine picks for this problem."""
    code = nat.load().dx_select_kernel(M, N, K, DTYPE_CODES[dtype])
    return {v: k for k, v in nat.KERNEL_NAMES.items()}[code]


def _ptr_array(ptrs):
    import ctypes
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    return arr


def reduce_broadcast(partial: torch.Tensor, p_ptrs, rank: int, rows_per_rank: int,
                     bias: torch.Tensor | None, residual: torch.Tensor | None, y_ptrs,
                     ldy: int) -> None:
    """This rank's rows of sum_s partial_s + bias + residual, written to every
    rank's output (dx_reduce_broadcast).  `partial` is this rank's partial
    buffer (its shape and dtype describe all of them); `p_ptrs` / `y_ptrs`
    are the peer-mapped addresses of every rank's partial / output buffer."""
    N = partial.shape[1]
    world = len(p_ptrs)
    lib = nat.load()
    with torch.cuda.device(partial.device):
        stream = torch.cuda.current_stream(partial.device).cuda_stream
        rc = lib.dx_reduce_broadcast(
            _ptr_array(p_ptrs), world, rank, rows_per_rank, N, _ld(partial),
            bias.data_ptr() if bias is not None else None,
            residual.data_ptr() if residual is not None else None,
            _ld(residual) if residual is not None else 0, _ptr_array(y_ptrs), ldy,
            DTYPE_CODES[partial.dtype], stream)
    nat.check("dx_reduce_broadcast", rc)


def row_flag_words() -> int:
    """int32 flag words each rank's flag buffer needs for a row-reduction job."""
    return int(nat.load().dx_row_flag_words())


def row_job(p_ptrs, s_ptrs, f_ptrs, rank: int, M: int, N: int, ldp: int,
            reduce_chunk: tuple[int, int, int] | None,
            gather_chunk: tuple[int, int, int] | None,
            bias: torch.Tensor | None, residual: torch.Tensor | None, out: torch.Tensor,
            epoch: int, dtype: torch.dtype, mc_part: int = 0, mc_out: int = 0,
            out_sym: torch.Tensor | None = None) -> "nat.RowReduceJob":
    """One job of the chunked row-parallel reduction (dx_row_reduce_job):
    reduce-scatter of `reduce_chunk` and all-gather of `gather_chunk`, each
    given as (first row, rows, chunk index) or None.  `p_ptrs` / `s_ptrs` /
    `f_ptrs` are the peer-mapped addresses of every rank's partial, slab and
    flag buffers; `out` is this rank's output.  With `mc_part` (the NVLink
    multicast address of the partial buffers) the job runs in the multicast
    form: `mc_out` / `out_sym` are the multicast address and this rank's view
    of the peer-written output buffer, and `s_ptrs` is unused."""
    j = nat.RowReduceJob()
    world = len(p_ptrs)
    for r in range(world):
        j.P[r], j.F[r] = p_ptrs[r], f_ptrs[r]
        j.S[r] = s_ptrs[r] if s_ptrs is not None else None
    j.world, j.rank, j.M, j.N, j.ldp = world, rank, M, N, ldp
    j.a_row0, j.a_rows, j.a_chunk = reduce_chunk if reduce_chunk is not None else (0, 0, 0)
    j.b_row0, j.b_rows, j.b_chunk = gather_chunk if gather_chunk is not None else (0, 0, 0)
    j.bias = bias.data_ptr() if bias is not None else None
    j.R = residual.data_ptr() if residual is not None else None
    j.ldr = _ld(residual) if residual is not None else 0
    j.Y, j.ldy = out.data_ptr(), _ld(out)
    j.epoch, j.dtype = epoch, DTYPE_CODES[dtype]
    if mc_part:
        j.mc_part, j.mc_out = mc_part, mc_out
        j.out_sym, j.ldo = out_sym.data_ptr(), _ld(out_sym)
    return j


def row_reduce(job: "nat.RowReduceJob", stream: int, grid: int = 0) -> None:
    """Run a row-reduction job as its own launch on `stream` (dx_row_reduce)."""
    nat.check("dx_row_reduce", nat.load().dx_row_reduce(ctypes.byref(job), grid, stream))
