"""ORACLE — test infrastructure only (tests/, __graft_entry__.smoke() and
bench.py's CPU baseline).  Nothing in the engine imports this package.

CPU restatements of the reference's fused-linear oracle
(deepx_op_gpukernelcompiler/kernel.py:64-66 with fusion.py:87-92):

    ref = act(a @ b + bias)           (+ residual for the MLP chain)

* ``fused_linear_f64`` — the C restatement in double precision
  (fused_linear_ref.c), for parity checks at test sizes;
* ``fused_linear_f32`` — numpy in fp32 (BLAS sgemm, then the epilogue),
  the same arithmetic class as the reference's torch-CPU fp32 oracle; used
  at sizes where the C loop would be slow and as the timed CPU baseline;
* ``mlp_residual_*`` — the two-GEMM chain H = act(X W1 + b1), Y = H W2 + b2 + X;
* ``gated_linear_f64`` / ``gated_ffn_f64`` — the gated FFN chain of
  fusion.py:44-46 (test/fusion_cases/07_ffn_gated.kv: tensor.silu of the gate
  GEMM, tensor.mul with the up GEMM, then the output GEMM), composed from the
  same restated matmul/add/activation steps.

Activations: relu; gelu = tanh approximation (fusion.py:89, the reference
oracle); gelu_erf = 0.5 x (1 + erf(x / sqrt 2)) (kernel_triton.py:61);
silu = swish = x * sigmoid(x) (fusion.py:90-91).
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from . import build_oracle

ACT_CODES = {None: 0, "none": 0, "relu": 1, "gelu": 2, "gelu_tanh": 2, "gelu_erf": 3,
             "silu": 4, "swish": 4}

_lib = None


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build_oracle.build()))
        dp = ctypes.POINTER(ctypes.c_double)
        lib.oracle_fused_linear_f64.restype = ctypes.c_int
        lib.oracle_fused_linear_f64.argtypes = [dp, dp, dp, dp, dp, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_int64, ctypes.c_int]
        lib.oracle_activation_f64.restype = ctypes.c_int
        lib.oracle_activation_f64.argtypes = [dp, dp, ctypes.c_int64, ctypes.c_int]
        _lib = lib
    return _lib


def _as_f64(a) -> np.ndarray | None:
    if a is None:
        return None
    if hasattr(a, "detach"):  # torch tensor (any dtype) -> exact fp64 values
        a = a.detach().cpu().double().numpy()
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def fused_linear_f64(X, W, bias=None, act=None, residual=None) -> np.ndarray:
    """act(X @ W + bias) + residual in double precision (C oracle)."""
    Xd, Wd, bd, Rd = _as_f64(X), _as_f64(W), _as_f64(bias), _as_f64(residual)
    M, K = Xd.shape
    K2, N = Wd.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {K} vs {K2}")
    if bd is not None and bd.shape != (N,):
        raise ValueError("bias shape")
    if Rd is not None and Rd.shape != (M, N):
        raise ValueError("residual shape")
    Y = np.empty((M, N), dtype=np.float64)
    rc = _load().oracle_fused_linear_f64(_ptr(Xd), _ptr(Wd), _ptr(bd), _ptr(Rd), _ptr(Y),
                                         M, N, K, ACT_CODES[act])
    if rc != 0:
        raise ValueError("oracle_fused_linear_f64 rejected its arguments")
    return Y


def activation_f64(x, act) -> np.ndarray:
    xd = _as_f64(x).reshape(-1)
    y = np.empty_like(xd)
    if _load().oracle_activation_f64(_ptr(xd), _ptr(y), xd.size, ACT_CODES[act]) != 0:
        raise ValueError("bad activation")
    return y.reshape(np.shape(_as_f64(x)))


_erf = np.vectorize(math.erf, otypes=[np.float64])


def _act_np(v: np.ndarray, act) -> np.ndarray:
    code = ACT_CODES[act]
    if code == 0:
        return v
    if code == 1:
        return np.maximum(v, np.float32(0))
    if code == 2:
        c = np.float32(math.sqrt(2.0 / math.pi))
        return (np.float32(0.5) * v * (np.float32(1) + np.tanh(c * (v + np.float32(0.044715) * v * v * v)))).astype(np.float32)
    if code == 3:
        try:
            from scipy.special import erf
            e = erf(v * np.float32(1 / math.sqrt(2.0))).astype(np.float32)
        except ImportError:  # pragma: no cover - scipy ships with the image
            e = _erf(v.astype(np.float64) / math.sqrt(2.0)).astype(np.float32)
        return (np.float32(0.5) * v * (np.float32(1) + e)).astype(np.float32)
    return (v / (np.float32(1) + np.exp(-v))).astype(np.float32)


def fused_linear_f32(X, W, bias=None, act=None, residual=None) -> np.ndarray:
    """act(X @ W + bias) + residual in fp32 with numpy (BLAS sgemm)."""
    def f32(a):
        if a is None:
            return None
        if hasattr(a, "detach"):
            a = a.detach().cpu().float().numpy()
        return np.asarray(a, dtype=np.float32)

    Xf, Wf, bf, Rf = f32(X), f32(W), f32(bias), f32(residual)
    Y = Xf @ Wf
    if bf is not None:
        Y += bf
    Y = _act_np(Y, act)
    if Rf is not None:
        Y += Rf
    return Y


def mlp_residual_f64(X, W1, b1, W2, b2, act="gelu") -> np.ndarray:
    """H = act(X W1 + b1), Y = H W2 + b2 + X, all in double (H not rounded)."""
    H = fused_linear_f64(X, W1, b1, act)
    return fused_linear_f64(H, W2, b2, None, residual=X)


def mlp_residual_f32(X, W1, b1, W2, b2, act="gelu") -> np.ndarray:
    H = fused_linear_f32(X, W1, b1, act)
    return fused_linear_f32(H, W2, b2, None, residual=X)


def gated_linear_f64(X, Wg, bg, Wu, bu, act="silu") -> np.ndarray:
    """act(X Wg + bg) * (X Wu + bu) in double precision (07_ffn_gated.kv:2-7)."""
    return fused_linear_f64(X, Wg, bg, act) * fused_linear_f64(X, Wu, bu, None)


def gated_ffn_f64(X, Wg, bg, Wu, bu, Wo, bo, act="silu") -> np.ndarray:
    """(act(X Wg + bg) * (X Wu + bu)) Wo + bo in double (07_ffn_gated.kv:2-9)."""
    return fused_linear_f64(gated_linear_f64(X, Wg, bg, Wu, bu, act), Wo, bo, None)


def gated_linear_f32(X, Wg, bg, Wu, bu, act="silu") -> np.ndarray:
    return fused_linear_f32(X, Wg, bg, act) * fused_linear_f32(X, Wu, bu, None)


def gated_ffn_f32(X, Wg, bg, Wu, bu, Wo, bo, act="silu") -> np.ndarray:
    return fused_linear_f32(gated_linear_f32(X, Wg, bg, Wu, bu, act), Wo, bo, None)
