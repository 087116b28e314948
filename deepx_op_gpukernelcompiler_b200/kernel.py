"""GPU kernel dispatcher + test/bench harness for compilable fusion patterns.

Same entry point and contract as the reference
(deepx_op_gpukernelcompiler/kernel.py:11-93): ``compile_and_test(kv, path)``
reads the function from kvspace, classifies it, runs the engine on random
fp16 inputs, compares with the PyTorch expression ``a @ b + bias`` ->
``ACTIVATION_PT[act]`` and times both (20 warm-up calls, then CUDA events
over 200 calls).  It returns ``CompileResult(success, diff, tl_ms, pt_ms,
error)`` with success = ``diff < 0.5``.

The only engine is the B200 one (``ENGINES = {"b200": ...}``): there is no
multi-backend dispatch and no CPU path.  Besides the compilable patterns it
runs the two single-GEMM patterns the reference lists as needs_template
(fusion.py:24-25): ``attention_output`` (template ``gemm``: a @ b) and
``attention_score`` (template ``gemm_elem``: (a @ b) * scale, with
scale = 1/sqrt(K)), through compiled plans (plan.py), and two of the
``multi_kernel`` FFN chains as chains of fused launches: ``ffn_two_layer``
(relu(a @ W1 + b1) @ W2 + b2, fusion.py:42-43) and ``ffn_gated``
((silu(a @ Wg + bg) * (a @ Wu + bu)) @ Wo + bo, fusion.py:44-46, the gate and
up GEMMs in one dual-GEMM launch).  Their weights are scaled by
1/sqrt(fan-in) so the chain's output stays O(1).  Extra keyword arguments over the
reference: ``dtype`` (default fp16 as in the reference), ``seed`` (default
unseeded, as in the reference), ``n_iter`` and ``warmup``.  ``block`` is
accepted for signature compatibility; the engine chooses its own tiles.
"""
from __future__ import annotations

import torch

from . import _native
from .fusion import ACTIVATION_PT, classify
from .kernel_b200 import make_linear_kernel
from .kvfunc import read_func
from .mlp import gated_ffn, mlp_residual, two_layer_ffn
from .plan import CompileRequest, Plan

DEFAULT_SHAPE = {"M": 512, "N": 512, "K": 256}
DEFAULT_BLOCK = {"BM": 128, "BN": 128, "BK": 32}

ENGINES = {
    "b200": make_linear_kernel,
}

# needs_template rows (fusion.py:24-25) whose template the engine implements.
ENGINE_TEMPLATES = {"gemm", "gemm_elem"}

# multi_kernel rows (fusion.py:42-46) the engine runs as chains of fused launches.
ENGINE_CHAINS = {"ffn_two_layer", "ffn_gated"}


class CompileResult:
    """Outcome of compile_and_test (kernel.py:20-27). ``tl_ms`` is the engine's time."""

    def __init__(self, success: bool, diff: float, tl_ms: float, pt_ms: float,
                 error: str | None = None):
        self.success = success
        self.diff = diff
        self.tl_ms = tl_ms
        self.pt_ms = pt_ms
        self.error = error

    def __repr__(self) -> str:
        return (f"CompileResult(success={self.success}, diff={self.diff:.6g}, "
                f"tl_ms={self.tl_ms:.4f}, pt_ms={self.pt_ms:.4f}, error={self.error!r})")


def _time_ms(fn, n_iter: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(n_iter):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / n_iter


def compile_and_test(kv, func_path: str, fusion: str = "b200", shape: dict | None = None,
                     block: dict | None = None, dtype: torch.dtype = torch.float16,
                     seed: int | None = None, n_iter: int = 200,
                     warmup: int = 20) -> CompileResult:
    """Read func from kvspace, run the fused engine, check and time it."""
    s = shape or DEFAULT_SHAPE
    M, N, K = s["M"], s["N"], s["K"]
    del block  # tile shapes are chosen by the engine

    func = read_func(kv, func_path)
    tensor_ops = [o for o in func["ops"] if o["op"] != "return"]
    pattern, template, activation, status = classify(func["ops"])
    if status == "not_matched":
        opcodes = " → ".join(o["op"] for o in tensor_ops)
        return CompileResult(False, 0, 0, 0, f"no fusion pattern for: {opcodes}")
    if status != "compilable" and template not in ENGINE_TEMPLATES and pattern not in ENGINE_CHAINS:
        return CompileResult(False, 0, 0, 0, f"{status}: {pattern}")
    if not torch.cuda.is_available():
        raise RuntimeError("compile_and_test needs a CUDA device (the B200 engine has no CPU path)")

    factory = ENGINES[fusion]
    dev = torch.device("cuda")
    gen = None
    if seed is not None:
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)

    def randn(*shape_):
        return torch.randn(shape_, dtype=dtype, device=dev, generator=gen)

    if template in ENGINE_TEMPLATES:
        a, b = randn(M, K), randn(K, N)
        scale = 1.0 / K ** 0.5 if template == "gemm_elem" else 1.0
        dtype_name = {torch.float16: "float16", torch.bfloat16: "bfloat16",
                      torch.float32: "float32"}[dtype]
        spec = {"pattern": pattern, "ops": [o["op"] for o in tensor_ops], "scale": scale,
                "inputs": [{"shape": [M, K], "dtype": dtype_name},
                           {"shape": [K, N], "dtype": dtype_name}]
                + ([{"shape": [1], "dtype": dtype_name}] if template == "gemm_elem" else []),
                "outputs": [{"shape": [M, N], "dtype": dtype_name}]}
        plan = Plan(CompileRequest.from_json(spec))

        def run():
            return plan(a, b)

        def ref_fn():
            out = a @ b
            return out * scale if template == "gemm_elem" else out
    elif pattern == "ffn_two_layer":
        # X[M,K] -> H[M,N] -> Y[M,K]
        a, w1, b1, w2, b2 = randn(M, K), randn(K, N), randn(N), randn(N, K), randn(K)
        w1 /= K ** 0.5
        w2 /= N ** 0.5

        def run():
            return two_layer_ffn(a, w1, b1, w2, b2, "relu")

        def ref_fn():
            return ACTIVATION_PT["relu"](a @ w1 + b1) @ w2 + b2
    elif pattern == "ffn_gated":
        # X[M,K] -> H[M,N] (gate * up) -> Y[M,K]
        a, wg, bg, wu, bu = randn(M, K), randn(K, N), randn(N), randn(K, N), randn(N)
        wo, bo = randn(N, K), randn(K)
        wg /= K ** 0.5
        wu /= K ** 0.5
        wo /= N ** 0.5

        def run():
            return gated_ffn(a, wg, bg, wu, bu, wo, bo, "silu")

        def ref_fn():
            return (ACTIVATION_PT["silu"](a @ wg + bg) * (a @ wu + bu)) @ wo + bo
    elif template == "mlp_chain":
        # X[M,K] -> H[M,N] -> Y[M,K]; residual is X itself.
        a, w1, b1, w2, b2 = randn(M, K), randn(K, N), randn(N), randn(N, K), randn(K)
        w1 /= K ** 0.5
        w2 /= N ** 0.5

        def run():
            return mlp_residual(a, w1, b1, w2, b2, activation or "gelu")

        def ref_fn():
            h = ACTIVATION_PT[activation or "gelu"](a @ w1 + b1)
            return h @ w2 + b2 + a
    else:
        kernel_fn = factory(activation)
        a, b, bias = randn(M, K), randn(K, N), randn(N)
        r = randn(M, N) if template == "linear_residual" else None

        def run():
            return kernel_fn(a, b, bias, residual=r)

        def ref_fn():
            out = a @ b + bias
            if activation and activation in ACTIVATION_PT:
                out = ACTIVATION_PT[activation](out)
            if r is not None:
                out = out + r
            return out

    out = run()
    torch.cuda.synchronize()
    ref = ref_fn()
    diff = (out.float() - ref.float()).abs().max().item()
    tl_ms = _time_ms(run, n_iter, warmup)
    pt_ms = _time_ms(ref_fn, n_iter, 0)
    # A launch whose bounded wait ran out leaves an incomplete output; the
    # timing loop has synchronised, so the status word is final here.
    status = _native.device_status(torch.cuda.current_stream().cuda_stream)
    if status:
        return CompileResult(False, diff, tl_ms, pt_ms,
                             f"device status {status}: a kernel gave up a bounded wait")
    return CompileResult(diff < 0.5, diff, tl_ms, pt_ms)
