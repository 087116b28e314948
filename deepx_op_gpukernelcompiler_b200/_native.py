"""ctypes binding of the C ABI in ``include/deepx_fused.h``.

The engine is a plain C-ABI shared library (``libdeepx_fused.so``, built
in-tree by ``_build.py``).  Python reaches it only through this module, with
raw device pointers, explicit leading dimensions and the current CUDA stream —
the same call a non-Python dispatcher makes (the docs' ``dlsym`` + raw pointer
runtime, doc/kernel-compiler-analysis.md:113-134).

There is no fallback: if the library is missing or fails to load, every
entry point raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdeepx_fused.so"

DX_OK = 0
DX_ERR_INVALID_ARGUMENT = -1
DX_ERR_UNSUPPORTED = -2
DX_ERR_CUDA = -3
DX_ERR_WORKSPACE = -4
DX_ERR_DEVICE_TIMEOUT = -5
ERROR_NAMES = {
    DX_ERR_INVALID_ARGUMENT: "DX_ERR_INVALID_ARGUMENT",
    DX_ERR_UNSUPPORTED: "DX_ERR_UNSUPPORTED",
    DX_ERR_CUDA: "DX_ERR_CUDA",
    DX_ERR_WORKSPACE: "DX_ERR_WORKSPACE",
    DX_ERR_DEVICE_TIMEOUT: "DX_ERR_DEVICE_TIMEOUT",
}

DX_DTYPE_F32 = 0
DX_DTYPE_F16 = 1
DX_DTYPE_BF16 = 2

DX_ACT_NONE = 0
DX_ACT_RELU = 1
DX_ACT_GELU_TANH = 2
DX_ACT_GELU_ERF = 3
DX_ACT_SILU = 4

DX_KERNEL_AUTO = 0
DX_KERNEL_UMMA = 1
DX_KERNEL_DECODE = 2
DX_KERNEL_SIMT = 3
DX_KERNEL_UMMA_1CTA = 4
KERNEL_NAMES = {"auto": DX_KERNEL_AUTO, "umma": DX_KERNEL_UMMA,
                "decode": DX_KERNEL_DECODE, "simt": DX_KERNEL_SIMT,
                "umma_1cta": DX_KERNEL_UMMA_1CTA}

DX_DEVICE_STATUS_TIMEOUT = 1

# Every function the header declares, with its ctypes signature.
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_LINEAR_ARGS = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                ctypes.c_int, ctypes.c_int]
SIGNATURES = {
    "dx_fused_linear": (ctypes.c_int, _LINEAR_ARGS + [_vp, ctypes.c_size_t, _vp]),
    "dx_fused_linear_ex": (ctypes.c_int, _LINEAR_ARGS + [ctypes.c_int, _vp, ctypes.c_size_t, _vp]),
    "dx_fused_linear_decode_noalloc": (ctypes.c_int, _LINEAR_ARGS + [_vp]),
    "dx_reduce_broadcast": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                           ctypes.c_int, _i64, _i64, _i64, _vp, _vp, _i64,
                                           ctypes.POINTER(ctypes.c_void_p), _i64, ctypes.c_int,
                                           _vp]),
    "dx_row_reduce": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, _vp]),
    "dx_fused_linear_rowjob": (ctypes.c_int, _LINEAR_ARGS + [ctypes.c_int, _vp, ctypes.c_size_t,
                                                             ctypes.c_void_p, _vp]),
    "dx_fused_gated_linear_rowjob": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                                    _i64, _i64, _i64, _i64, _i64, ctypes.c_int,
                                                    ctypes.c_int, ctypes.c_int, _vp,
                                                    ctypes.c_size_t, ctypes.c_void_p, _vp]),
    "dx_row_flag_words": (ctypes.c_int, []),
    "dx_fused_linear_workspace_size": (ctypes.c_size_t, [_i64, _i64, _i64, ctypes.c_int, ctypes.c_int]),
    "dx_fused_gated_linear": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                             _i64, _i64, _i64, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, _vp, ctypes.c_size_t, _vp]),
    "dx_fused_gated_linear_workspace_size": (ctypes.c_size_t, [_i64, _i64, _i64, ctypes.c_int,
                                                               ctypes.c_int]),
    "dx_select_kernel": (ctypes.c_int, [_i64, _i64, _i64, ctypes.c_int]),
    "dx_copy_2d_async": (ctypes.c_int, [_vp, ctypes.c_size_t, _vp, ctypes.c_size_t,
                                        ctypes.c_size_t, ctypes.c_size_t, _vp]),
    "dx_last_error_string": (ctypes.c_char_p, []),
    "dx_last_launch_plan": (ctypes.c_char_p, []),
    "dx_set_trace_buffer": (ctypes.c_int, [_vp, ctypes.c_size_t]),
    "dx_device_status": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int)]),
    "dx_version": (ctypes.c_int, []),
    "dx_kernel_arch": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "dx_selftest_bounded_wait": (ctypes.c_int, [_vp, _vp]),
    "dx_plan_create": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), _i64, _i64, _i64,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int]),
    "dx_plan_workspace_size": (ctypes.c_size_t, [_vp]),
    "dx_plan_set_workspace": (ctypes.c_int, [_vp, _vp, ctypes.c_size_t]),
    "dx_plan_call": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "dx_plan_call_residual": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "dx_plan_destroy": (ctypes.c_int, [_vp]),
}



class RowReduceJob(ctypes.Structure):
    """ctypes mirror of ``dx_row_reduce_job`` (include/deepx_fused.h)."""

    _fields_ = [
        ("P", ctypes.c_void_p * 8),
        ("S", ctypes.c_void_p * 8),
        ("F", ctypes.c_void_p * 8),
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("M", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("ldp", ctypes.c_int64),
        ("a_row0", ctypes.c_int64),
        ("a_rows", ctypes.c_int64),
        ("a_chunk", ctypes.c_int),
        ("b_row0", ctypes.c_int64),
        ("b_rows", ctypes.c_int64),
        ("b_chunk", ctypes.c_int),
        ("bias", ctypes.c_void_p),
        ("R", ctypes.c_void_p),
        ("ldr", ctypes.c_int64),
        ("Y", ctypes.c_void_p),
        ("ldy", ctypes.c_int64),
        ("epoch", ctypes.c_int),
        ("dtype", ctypes.c_int),
        ("mc_part", ctypes.c_void_p),
        ("mc_out", ctypes.c_void_p),
        ("out_sym", ctypes.c_void_p),
        ("ldo", ctypes.c_int64),
    ]


_lock = threading.Lock()
_lib = None


class NativeError(RuntimeError):
    """A C-ABI call returned a negative DX_ERR_* code."""

    def __init__(self, func: str, code: int, message: str):
        self.code = code
        super().__init__(f"{func} failed with {ERROR_NAMES.get(code, code)}: {message}")


def load() -> ctypes.CDLL:
    """Load (once) and return the engine library; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"native engine {LIB_PATH.name} is not built; run "
                    "`python -m deepx_op_gpukernelcompiler_b200._build` (needs nvcc)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def last_error() -> str:
    return load().dx_last_error_string().decode("utf-8", "replace")


def last_launch_plan() -> str:
    """Kernel variant, tiling and grid of the last launch on this thread."""
    return load().dx_last_launch_plan().decode("utf-8", "replace")


def check(func: str, rc: int) -> None:
    if rc != DX_OK:
        raise NativeError(func, rc, last_error())


def device_status(stream: int = 0) -> int:
    """Synchronise `stream` and return (and clear) the device status bits."""
    st = ctypes.c_int(0)
    check("dx_device_status", load().dx_device_status(stream, ctypes.byref(st)))
    return st.value
