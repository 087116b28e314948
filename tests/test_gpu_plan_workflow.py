"""Plans and the reference-facing harness on the GPU (gpu).

* compiled plans (the docs' compile request -> ``call(x, W, b, out, stream)``)
  for every plannable pattern, against the fp64 oracle;
* ``compile_and_test`` — the reference's harness (kernel.py:30-93) — on every
  runnable function of the package's ``.kv`` fixtures, and the workflow CLI
  over all of them.
"""
from pathlib import Path

import pytest
import torch

import deepx_op_gpukernelcompiler_b200 as pkg
import oracle
from deepx_op_gpukernelcompiler_b200 import compile_and_test, kvload, workflow
from deepx_op_gpukernelcompiler_b200.kvspace_local import KVSpace
from deepx_op_gpukernelcompiler_b200.plan import PlanCache

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
KV_DIR = Path(pkg.__file__).parent / "kv"


def _request(pattern, ops, M, K, N, dtype="bfloat16", extra_inputs=(), scale=None):
    req = {"pattern": pattern, "ops": ops,
           "inputs": [{"shape": [M, K], "dtype": dtype}, {"shape": [K, N], "dtype": dtype},
                      *extra_inputs],
           "outputs": [{"shape": [M, N], "dtype": dtype}]}
    if scale is not None:
        req["scale"] = scale
    return req


@pytest.mark.parametrize("pattern,ops,act", [
    ("linear", ["matmul", "add"], None),
    ("linear_relu", ["matmul", "add", "relu"], "relu"),
    ("linear_gelu", ["matmul", "add", "gelu"], "gelu"),
    ("linear_silu", ["matmul", "add", "silu"], "silu"),
    ("linear_swish", ["matmul", "add", "swish"], "silu"),
])
@pytest.mark.parametrize("M", [16, 300])
def test_linear_plans(pattern, ops, act, M):
    K, N = 512, 384
    cache = PlanCache()
    plan = cache.get(_request(pattern, ops, M, K, N, extra_inputs=[{"shape": [N], "dtype": "bfloat16"}]))
    g = torch.Generator().manual_seed(M)
    X = torch.randn(M, K, generator=g).bfloat16()
    W = (torch.randn(K, N, generator=g) / K ** 0.5).bfloat16()
    b = (torch.rand(N, generator=g) * 0.2 - 0.1).bfloat16()
    Y = plan(X.to(DEV), W.to(DEV), b.to(DEV))
    torch.cuda.synchronize()
    ref = torch.from_numpy(oracle.fused_linear_f64(X, W, b, act)).float()
    assert torch.allclose(Y.float().cpu(), ref, rtol=2e-2, atol=2e-2)


def test_residual_and_gemm_template_plans():
    M, K, N = 256, 256, 256
    g = torch.Generator().manual_seed(3)
    X = torch.randn(M, K, generator=g).half()
    W = (torch.randn(K, N, generator=g) / K ** 0.5).half()
    b = (torch.rand(N, generator=g) * 0.2 - 0.1).half()
    R = torch.randn(M, N, generator=g).half()
    cache = PlanCache()
    f16 = "float16"
    res = cache.get(_request("linear_residual", ["matmul", "add", "add"], M, K, N, f16,
                             [{"shape": [N], "dtype": f16}, {"shape": [M, N], "dtype": f16}]))
    Y = res(X.to(DEV), W.to(DEV), b.to(DEV), residual=R.to(DEV))
    out = cache.get(_request("attention_output", ["matmul"], M, K, N, f16))
    Yo = out(X.to(DEV), W.to(DEV))
    score = cache.get(_request("attention_score", ["matmul", "mul"], M, K, N, f16,
                               [{"shape": [1], "dtype": f16}], scale=0.0625))
    Ys = score(X.to(DEV), W.to(DEV))
    torch.cuda.synchronize()
    for got, ref in ((Y, oracle.fused_linear_f64(X, W, b, None, residual=R)),
                     (Yo, oracle.fused_linear_f64(X, W, None, None)),
                     (Ys, 0.0625 * oracle.fused_linear_f64(X, W, None, None))):
        assert torch.allclose(got.float().cpu(), torch.from_numpy(ref).float(), rtol=2e-2, atol=2e-2)


@pytest.fixture(scope="module")
def kv():
    store = KVSpace()
    kvload.load_dir(store, KV_DIR, pkg="fusion_cases")
    return store


@pytest.mark.parametrize("name", ["dense", "dense_relu", "dense_gelu", "dense_silu", "dense_swish",
                                  "dense_residual", "mlp_block", "scaled_scores",
                                  "two_layer_relu", "gated_silu"])
def test_compile_and_test_runs_engine(kv, name):
    r = compile_and_test(kv, f"/func/fusion_cases/{name}", seed=0, n_iter=5, warmup=2)
    assert r.error is None and r.success, r
    assert r.tl_ms > 0 and r.pt_ms > 0


def test_workflow_all(capsys):
    workflow.main(["--load", str(KV_DIR), "--all"])
    out = capsys.readouterr().out
    assert "summary" in out and "compilable: 7" in out


def test_mlp_residual_chain_plan_and_record():
    """cfg5's pattern through the compile-then-call runtime: two native plans
    (dx_plan_call, then dx_plan_call_residual with X as the residual), and a
    kvspace record that lists both calls for a non-Python dispatcher."""
    M, K, H = 512, 256, 1024
    dt = "bfloat16"
    req = {"func": "mlp_block", "pattern": "mlp_residual",
           "ops": ["matmul", "add", "gelu", "matmul", "add", "add"],
           "inputs": [{"shape": s, "dtype": dt} for s in ([M, K], [K, H], [H], [H, K], [K])],
           "outputs": [{"shape": [M, K], "dtype": dt}]}
    store = KVSpace()
    cache = PlanCache(store)
    plan = cache.get(req)
    g = torch.Generator().manual_seed(41)
    X = torch.randn(M, K, generator=g).bfloat16()
    W1 = (torch.randn(K, H, generator=g) / K ** 0.5).bfloat16()
    b1 = (torch.rand(H, generator=g) * 0.2 - 0.1).bfloat16()
    W2 = (torch.randn(H, K, generator=g) / H ** 0.5).bfloat16()
    b2 = (torch.rand(K, generator=g) * 0.2 - 0.1).bfloat16()
    Y = plan(X.to(DEV), W1.to(DEV), b1.to(DEV), W2.to(DEV), b2.to(DEV))
    torch.cuda.synchronize()
    ref = oracle.mlp_residual_f64(X, W1, b1, W2, b2, "gelu")
    assert torch.allclose(Y.float().cpu(), torch.from_numpy(ref).float(), rtol=2e-2, atol=2e-2)
    (record,) = cache.records("mlp_block").values()
    assert [c["entry"] for c in record["calls"]] == ["dx_plan_call", "dx_plan_call_residual"]
    assert cache.get(req) is plan and cache.hits == 1
