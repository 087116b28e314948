"""B200-native engine for DeepX's fused-op compiler hot path.

Public surface, as the reference package (deepx_op_gpukernelcompiler/
__init__.py:1-3): ``read_func, list_funcs, FUSION_DB, classify,
ACTIVATION_PT, compile_and_test, CompileResult, ENGINES``, plus the engine
itself: ``make_linear_kernel`` (the factory registered in ``ENGINES``),
``fused_linear`` (tensor-level call), ``fused_linear_host`` (host buffers,
copies overlapped with the fused launches), ``fused_gated_linear`` (the gated
dual GEMM) and the FFN chains ``mlp_residual``, ``gated_ffn`` and
``two_layer_ffn``.  Every compute call goes through the C ABI of
``libdeepx_fused.so`` (include/deepx_fused.h).
"""
from .fusion import ACTIVATION_PT, FUSION_DB, classify
from .kernel import ENGINES, CompileResult, compile_and_test
from .kernel_b200 import make_linear_kernel
from .kvfunc import list_funcs, read_func
from .linear import fused_gated_linear, fused_linear, fused_linear_host
from .mlp import gated_ffn, mlp_residual, two_layer_ffn

__all__ = [
    "read_func", "list_funcs", "FUSION_DB", "classify", "ACTIVATION_PT",
    "compile_and_test", "CompileResult", "ENGINES",
    "make_linear_kernel", "fused_linear", "fused_linear_host", "fused_gated_linear",
    "mlp_residual", "gated_ffn",
    "two_layer_ffn",
]
