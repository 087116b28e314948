"""Fusion pattern database: kvlang opcode chains -> kernel templates.

The table and ``classify`` keep the reference's interface and contents
(deepx_op_gpukernelcompiler/fusion.py:14-109): the key is the exact tuple of
``tensor.*`` opcodes of a function (``return`` dropped), the value is
``(pattern_name, template_key, status)`` with status one of

    compilable      one fused kernel exists for the chain
    needs_template  one kernel would do, but no template exists
    multi_kernel    needs several kernels (two or more GEMMs)
    not_fusable     no GEMM+epilogue form

The reference rows are kept as they are (same keys, same values) so that a
function classifies identically under both packages.  Two rows are added for
chains the B200 engine runs in fused form and the reference has no entry for:

    matmul -> add -> add                       linear_residual  (Y = XW + b + R)
    matmul -> add -> gelu -> matmul -> add -> add
                                               mlp_residual     (two fused
                                               launches: H = GELU(XW1+b1),
                                               Y = HW2 + b2 + X)
"""
from __future__ import annotations

import torch

COMPILABLE = "compilable"
NEEDS_TEMPLATE = "needs_template"
MULTI_KERNEL = "multi_kernel"
NOT_FUSABLE = "not_fusable"
NOT_MATCHED = "not_matched"


def _chain(ops: str) -> tuple:
    return tuple(f"tensor.{op}" for op in ops.split())


# (opcode chain, pattern, template, status) — reference rows, fusion.py:14-85.
_REFERENCE_ROWS = [
    # one GEMM + elementwise epilogue
    ("matmul add", "linear", "linear", COMPILABLE),
    ("matmul add relu", "linear_relu", "linear_activation", COMPILABLE),
    ("matmul add gelu", "linear_gelu", "linear_activation", COMPILABLE),
    ("matmul add silu", "linear_silu", "linear_activation", COMPILABLE),
    ("matmul add swish", "linear_swish", "linear_activation", COMPILABLE),
    # single kernel possible, no template
    ("matmul mul", "attention_score", "gemm_elem", NEEDS_TEMPLATE),
    ("matmul", "attention_output", "gemm", NEEDS_TEMPLATE),
    ("add softmax", "attention_softmax", "softmax", NEEDS_TEMPLATE),
    ("mean sub square mean add sqrt div mul add", "layernorm", "norm", NEEDS_TEMPLATE),
    ("square mean add rsqrt mul mul", "rmsnorm", "norm", NEEDS_TEMPLATE),
    ("sub add sqrt div mul add", "batchnorm", "norm", NEEDS_TEMPLATE),
    ("reshape mean sub square mean add sqrt div mul add", "groupnorm", "norm", NEEDS_TEMPLATE),
    ("add square mean add rsqrt mul mul", "residual_add_norm", "norm", NEEDS_TEMPLATE),
    # two or more GEMMs
    ("matmul add relu matmul add", "ffn_two_layer", None, MULTI_KERNEL),
    ("matmul add silu matmul add mul matmul add", "ffn_gated", None, MULTI_KERNEL),
    ("matmul add gelu matmul add gelu matmul add", "ffn_sequential", None, MULTI_KERNEL),
    ("matmul add softmax matmul add mul matmul add", "moe_ffn", None, MULTI_KERNEL),
    ("matmul add matmul add matmul add", "qkv_projection", None, MULTI_KERNEL),
    ("matmul add matmul add matmul softmax matmul add matmul add", "mha_forward", None,
     MULTI_KERNEL),
    ("matmul add matmul matmul mul add", "lora_forward", None, MULTI_KERNEL),
    ("conv2d add relu conv2d add add relu", "resnet_block", None, MULTI_KERNEL),
    ("matmul add matmul add scatter scatter", "kv_cache_update", None, MULTI_KERNEL),
    ("mean sub square mean add rsqrt mul mul add matmul add", "pre_norm_linear", None,
     MULTI_KERNEL),
    # not GEMM + epilogue
    ("conv2d add", "conv2d", None, NOT_FUSABLE),
    ("conv2d add relu", "conv2d_relu", None, NOT_FUSABLE),
    ("conv2d sub add rsqrt mul mul add relu", "conv_bn_relu", None, NOT_FUSABLE),
    ("conv2d_dw add relu conv2d add", "depthwise_conv", None, NOT_FUSABLE),
    ("embedding", "embedding_lookup", None, NOT_FUSABLE),
    ("log_softmax nll_loss", "cross_entropy", None, NOT_FUSABLE),
]

# Chains the B200 engine adds (no reference row matches them).
_EXTENSION_ROWS = [
    ("matmul add add", "linear_residual", "linear_residual", COMPILABLE),
    ("matmul add gelu matmul add add", "mlp_residual", "mlp_chain", COMPILABLE),
]

REFERENCE_DB = {_chain(ops): (pat, tpl, st) for ops, pat, tpl, st in _REFERENCE_ROWS}
EXTENSION_DB = {_chain(ops): (pat, tpl, st) for ops, pat, tpl, st in _EXTENSION_ROWS}
FUSION_DB = {**REFERENCE_DB, **EXTENSION_DB}

ACTIVATIONS = ("relu", "gelu", "silu", "swish")

# PyTorch definitions of the activations (fusion.py:87-92): GELU is the tanh
# approximation, swish is SiLU.  gelu_erf is the exact form the reference's
# kernels compute (kernel_triton.py:61).
ACTIVATION_PT = {
    "relu": lambda t: torch.relu(t),
    "gelu": lambda t: torch.nn.functional.gelu(t, approximate="tanh"),
    "silu": lambda t: torch.nn.functional.silu(t),
    "swish": lambda t: torch.nn.functional.silu(t),
    "gelu_tanh": lambda t: torch.nn.functional.gelu(t, approximate="tanh"),
    "gelu_erf": lambda t: torch.nn.functional.gelu(t, approximate="none"),
}


def classify(ops: list) -> tuple:
    """Match an op list -> ``(pattern, template, activation, status)``.

    As fusion.py:95-109: ``return`` is ignored, the opcode tuple must match a
    row exactly, and only compilable rows report an activation.  The
    activation is the chain's activation opcode (relu/gelu/silu/swish); for
    the reference rows that is always the last opcode, so results agree with
    the reference, and for ``mlp_residual`` it is the inner GELU.
    """
    tensor_ops = [o for o in ops if o["op"] != "return"]
    opcodes = tuple(o["op"] for o in tensor_ops)
    row = FUSION_DB.get(opcodes)
    if row is None:
        return None, None, None, NOT_MATCHED
    pattern, template, status = row
    if status != COMPILABLE:
        return pattern, template, None, status
    activation = None
    for op in opcodes:
        name = op[len("tensor."):] if op.startswith("tensor.") else op
        if name in ACTIVATIONS:
            activation = name
    return pattern, template, activation, status
