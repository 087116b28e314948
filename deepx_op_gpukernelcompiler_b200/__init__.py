"""B200-native engine for DeepX's fused-op compiler hot path.

Public surface, as the reference package (deepx_op_gpukernelcompiler/
__init__.py:1-3): ``read_func, list_funcs, FUSION_DB, classify,
ACTIVATION_PT, compile_and_test, CompileResult, ENGINES``, plus the engine
itself: ``make_linear_kernel`` (the factory registered in ``ENGINES``),
``fused_linear`` (tensor-level call) and ``mlp_residual`` (the two-GEMM
chain).  Every compute call goes through the C ABI of
``libdeepx_fused.so`` (include/deepx_fused.h).
"""
from .fusion import ACTIVATION_PT, FUSION_DB, classify
from .kernel import ENGINES, CompileResult, compile_and_test
from .kernel_b200 import make_linear_kernel
from .kvfunc import list_funcs, read_func
from .linear import fused_linear
from .mlp import mlp_residual

__all__ = [
    "read_func", "list_funcs", "FUSION_DB", "classify", "ACTIVATION_PT",
    "compile_and_test", "CompileResult", "ENGINES",
    "make_linear_kernel", "fused_linear", "mlp_residual",
]
