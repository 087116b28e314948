"""The C-ABI library: loads, exports every declared symbol, and rejects bad
arguments on the host before touching a device (CPU; no compute calls)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from deepx_op_gpukernelcompiler_b200 import _build, _native as nat
from deepx_op_gpukernelcompiler_b200 import fused_linear, make_linear_kernel

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def lib():
    _build.build()
    return nat.load()


def _declared_functions() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"^\s*(?:const\s+)?[\w]+\s*\*?\s*(dx_\w+)\s*\(", text, re.M))
    return names


def test_every_declared_symbol_is_exported(lib):
    declared = _declared_functions()
    assert {"dx_fused_linear", "dx_fused_linear_ex", "dx_last_error_string"} <= declared
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert declared == set(nat.SIGNATURES), "ctypes signatures out of sync with the header"


def test_library_is_built_for_sm100a_only():
    """The build compiles one target, sm_100a (the run-time check of the
    loaded kernels' architecture is test_gpu_parity's dx_kernel_arch test)."""
    from deepx_op_gpukernelcompiler_b200 import _build
    assert _build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_version(lib):
    assert lib.dx_version() == 100


def _call(lib, **kw):
    args = dict(X=None, W=None, bias=None, R=None, Y=None, M=4, N=4, K=4, ldx=4, ldw=4, ldr=0,
                ldy=4, dtype=nat.DX_DTYPE_BF16, act=0, kernel=0, ws=None, ws_bytes=0, stream=None)
    args.update(kw)
    return lib.dx_fused_linear_ex(args["X"], args["W"], args["bias"], args["R"], args["Y"],
                                  args["M"], args["N"], args["K"], args["ldx"], args["ldw"],
                                  args["ldr"], args["ldy"], args["dtype"], args["act"],
                                  args["kernel"], args["ws"], args["ws_bytes"], args["stream"])


FAKE = 0x1000  # never dereferenced: validation fails first


@pytest.mark.parametrize("kw,code,needle", [
    (dict(dtype=7), nat.DX_ERR_INVALID_ARGUMENT, "dtype"),
    (dict(act=9), nat.DX_ERR_INVALID_ARGUMENT, "activation"),
    (dict(kernel=5), nat.DX_ERR_INVALID_ARGUMENT, "kernel"),
    (dict(M=-1), nat.DX_ERR_INVALID_ARGUMENT, "negative"),
    (dict(M=1 << 40), nat.DX_ERR_UNSUPPORTED, "2^31"),
    (dict(Y=None, X=FAKE, W=FAKE), nat.DX_ERR_INVALID_ARGUMENT, "Y is NULL"),
    (dict(Y=FAKE), nat.DX_ERR_INVALID_ARGUMENT, "X or W"),
    (dict(X=FAKE, W=FAKE, Y=FAKE, ldx=3), nat.DX_ERR_INVALID_ARGUMENT, "ldx"),
    (dict(X=FAKE, W=FAKE, Y=FAKE, ldw=2), nat.DX_ERR_INVALID_ARGUMENT, "ldw"),
    (dict(X=FAKE, W=FAKE, Y=FAKE, ldy=1), nat.DX_ERR_INVALID_ARGUMENT, "ldy"),
    (dict(X=FAKE, W=FAKE, Y=FAKE, R=FAKE, ldr=2), nat.DX_ERR_INVALID_ARGUMENT, "ldr"),
])
def test_host_validation(lib, kw, code, needle):
    assert _call(lib, **kw) == code
    assert needle in nat.last_error()


def _call_gated(lib, **kw):
    a = dict(X=FAKE, Wg=FAKE, Wu=FAKE, bg=None, bu=None, Y=FAKE, M=4, N=4, K=4, ldx=4, ldwg=4,
             ldwu=4, ldy=4, dtype=nat.DX_DTYPE_BF16, act=nat.DX_ACT_SILU, kernel=0)
    a.update(kw)
    return lib.dx_fused_gated_linear(a["X"], a["Wg"], a["Wu"], a["bg"], a["bu"], a["Y"], a["M"],
                                     a["N"], a["K"], a["ldx"], a["ldwg"], a["ldwu"], a["ldy"],
                                     a["dtype"], a["act"], a["kernel"], None, 0, None)


@pytest.mark.parametrize("kw,code,needle", [
    (dict(Wu=None), nat.DX_ERR_INVALID_ARGUMENT, "Wu is NULL"),
    (dict(ldwu=3), nat.DX_ERR_INVALID_ARGUMENT, "ldwu"),
    (dict(ldwg=3), nat.DX_ERR_INVALID_ARGUMENT, "ldw"),
    (dict(act=11), nat.DX_ERR_INVALID_ARGUMENT, "activation"),
    (dict(kernel=9), nat.DX_ERR_INVALID_ARGUMENT, "kernel"),
])
def test_gated_host_validation(lib, kw, code, needle):
    assert _call_gated(lib, **kw) == code
    assert needle in nat.last_error()


def test_gated_workspace_sizes(lib):
    # No GPU here: the device-dependent decode size reads as 0; the tensor-core
    # and SIMT forms never need one.
    assert lib.dx_fused_gated_linear_workspace_size(4096, 4096, 4096, nat.DX_DTYPE_BF16,
                                                    nat.DX_KERNEL_UMMA) == 0
    assert lib.dx_fused_gated_linear_workspace_size(16, 512, 512, nat.DX_DTYPE_F32, 0) == 0


def test_copy_2d_validation(lib):
    assert lib.dx_copy_2d_async(None, 0, None, 0, 0, 5, None) == nat.DX_OK  # empty
    assert lib.dx_copy_2d_async(FAKE, 8, FAKE, 16, 16, 2, None) == nat.DX_ERR_INVALID_ARGUMENT
    assert "pitch" in nat.last_error()
    assert lib.dx_copy_2d_async(None, 16, FAKE, 16, 16, 2, None) == nat.DX_ERR_INVALID_ARGUMENT


def test_host_entry_rejects_device_or_mismatched_tensors():
    from deepx_op_gpukernelcompiler_b200 import fused_linear_host
    X = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="host tensor"):
        fused_linear_host(X, torch.zeros(8, 4, dtype=torch.float16))
    with pytest.raises(ValueError, match="bias"):
        fused_linear_host(X, torch.zeros(8, 4, dtype=torch.bfloat16),
                          torch.zeros(3, dtype=torch.bfloat16))



def test_host_entry_load_order():
    """The host-buffer entry copies X's row blocks and W's column blocks in an
    expanding square (the next row block while the loaded columns are at
    least as wide as the loaded rows are tall), each block exactly once."""
    from deepx_op_gpukernelcompiler_b200.linear import _block_bounds, _load_order
    rows, cols = _block_bounds(8192, 8, 256), _block_bounds(14336, 8, 256)
    order = _load_order(rows, cols)
    assert order[:4] == [("r", 0), ("c", 0), ("r", 1), ("c", 1)]
    assert sorted(i for k, i in order if k == "r") == list(range(8))
    assert sorted(i for k, i in order if k == "c") == list(range(8))
    tall = wide = 0
    for k, i in order[:-1]:  # the loaded region stays near-square
        tall += rows[i][1] - rows[i][0] if k == "r" else 0
        wide += cols[i][1] - cols[i][0] if k == "c" else 0
        if tall and wide:
            assert max(tall, wide) <= 2 * min(tall, wide) + 1792
    assert _load_order(_block_bounds(512, 1, 256), _block_bounds(512, 1, 256)) == [("r", 0), ("c", 0)]
    assert _load_order(_block_bounds(4096, 4, 256), _block_bounds(256, 1, 256))[-1] == ("r", 3)

def test_empty_problem_is_a_no_op(lib):
    assert _call(lib, M=0) == nat.DX_OK
    assert _call(lib, N=0) == nat.DX_OK
    assert nat.last_error() == ""


def test_kernel_selection(lib):
    assert lib.dx_select_kernel(256, 512, 512, nat.DX_DTYPE_F32) == nat.DX_KERNEL_SIMT
    assert lib.dx_select_kernel(16, 28672, 8192, nat.DX_DTYPE_F16) == nat.DX_KERNEL_DECODE
    assert lib.dx_select_kernel(1, 3584, 8192, nat.DX_DTYPE_F16) == nat.DX_KERNEL_DECODE
    # M = 16 with fewer than 20 tiles: the tensor-core kernel only for the
    # smallest W (K * N < 2^23); M < 16 always streams through the decode kernel
    assert lib.dx_select_kernel(16, 1792, 4096, nat.DX_DTYPE_F16) == nat.DX_KERNEL_UMMA
    assert lib.dx_select_kernel(12, 1792, 4096, nat.DX_DTYPE_F16) == nat.DX_KERNEL_DECODE
    assert lib.dx_select_kernel(16, 3584, 8192, nat.DX_DTYPE_F16) == nat.DX_KERNEL_DECODE
    assert lib.dx_select_kernel(16, 7168, 8192, nat.DX_DTYPE_F16) == nat.DX_KERNEL_DECODE
    # 16 < M <= 32: decode only when W has >= SMs/2 tiles of 256 columns
    assert lib.dx_select_kernel(32, 28672, 8192, nat.DX_DTYPE_F16) == nat.DX_KERNEL_DECODE
    assert lib.dx_select_kernel(32, 3584, 8192, nat.DX_DTYPE_F16) == nat.DX_KERNEL_UMMA
    # 32 < M <= 64: the single-CTA tensor-core kernel streams W faster
    assert lib.dx_select_kernel(64, 28672, 8192, nat.DX_DTYPE_BF16) == nat.DX_KERNEL_UMMA
    assert lib.dx_select_kernel(8192, 14336, 4096, nat.DX_DTYPE_BF16) == nat.DX_KERNEL_UMMA
    assert lib.dx_select_kernel(8192, 14336, 4095, nat.DX_DTYPE_BF16) == nat.DX_KERNEL_SIMT
    assert lib.dx_select_kernel(64, 100, 0, nat.DX_DTYPE_BF16) == nat.DX_KERNEL_SIMT


def test_workspace_is_zero_when_not_needed(lib):
    assert lib.dx_fused_linear_workspace_size(8192, 14336, 4096, nat.DX_DTYPE_BF16,
                                              nat.DX_KERNEL_UMMA) == 0
    assert lib.dx_fused_linear_workspace_size(16, 512, 512, nat.DX_DTYPE_F32, 0) == 0


def test_error_string_is_thread_local(lib):
    import threading
    _call(lib, dtype=7)
    seen = {}

    def worker():
        seen["other"] = nat.last_error()

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert seen["other"] == ""
    assert "dtype" in nat.last_error()


def test_native_error_carries_code(lib):
    with pytest.raises(nat.NativeError) as ei:
        nat.check("dx_fused_linear", _call(lib, act=9))
    assert ei.value.code == nat.DX_ERR_INVALID_ARGUMENT


def test_wrapper_rejects_cpu_tensors():
    with pytest.raises(ValueError, match="CUDA"):
        fused_linear(torch.zeros(4, 4), torch.zeros(4, 4))


def test_wrapper_rejects_unknown_activation():
    with pytest.raises(ValueError, match="activation"):
        make_linear_kernel("tanh")
    with pytest.raises(ValueError, match="kernel"):
        fused_linear(torch.zeros(4, 4), torch.zeros(4, 4), kernel="cublas")


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(nat, "_lib", None)
    monkeypatch.setattr(nat, "LIB_PATH", tmp_path / "absent.so")
    with pytest.raises(RuntimeError, match="not built"):
        nat.load()


def test_ctypes_types_match_header(lib):
    assert lib.dx_fused_linear.restype is ctypes.c_int
    assert lib.dx_fused_linear_workspace_size.restype is ctypes.c_size_t


def test_row_reduce_job_layout_matches_header(tmp_path):
    """The ctypes mirror of dx_row_reduce_job has the C compiler's layout."""
    import shutil
    import subprocess
    from pathlib import Path
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f for f, _ in nat.RowReduceJob._fields_]
    src = tmp_path / "layout.c"
    body = "".join(f'printf("{f} %zu\\n", offsetof(dx_row_reduce_job, {f}));' for f in fields)
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "deepx_fused.h"\n'
                   'int main(void) {' + body +
                   'printf("size %zu\\n", sizeof(dx_row_reduce_job)); return 0; }\n')
    include = Path(__file__).resolve().parent.parent / "include"
    exe = tmp_path / "layout"
    subprocess.run([cc, f"-I{include}", str(src), "-o", str(exe)], check=True)
    got = dict(line.split() for line in subprocess.run(
        [str(exe)], check=True, capture_output=True, text=True).stdout.splitlines())
    for f in fields:
        assert int(got[f]) == getattr(nat.RowReduceJob, f).offset, f
    assert int(got["size"]) == ctypes.sizeof(nat.RowReduceJob)
