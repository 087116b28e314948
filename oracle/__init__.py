"""ORACLE — test infrastructure only.

CPU restatements of the reference's fused-linear oracle used to check the
engine.  Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline
may import this package; the engine never does.
"""
from .fused_linear import (  # noqa: F401
    ACT_CODES,
    activation_f64,
    fused_linear_f32,
    fused_linear_f64,
    gated_ffn_f32,
    gated_ffn_f64,
    gated_linear_f32,
    gated_linear_f64,
    mlp_residual_f32,
    mlp_residual_f64,
)
from . import torch_cpu  # noqa: F401,E402
