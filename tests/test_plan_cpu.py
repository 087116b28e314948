"""Compile requests and plans: parsing, validation and the plan cache (CPU).

The request format is the reference docs' JSON compile request
(doc/kvlang-to-tilelang-interface.md:100-129); creating a native plan is
host-only, so the cache is exercised without a GPU.
"""
import json

import pytest
import torch

from deepx_op_gpukernelcompiler_b200 import _build
from deepx_op_gpukernelcompiler_b200.plan import CompileError, CompileRequest, PlanCache

DOC_REQUEST = {
    "func": "__fusion_0", "pattern": "linear_relu", "ops": ["matmul", "add", "relu"],
    "inputs": [{"shape": [512, 256], "dtype": "float16"},
               {"shape": [256, 512], "dtype": "float16"},
               {"shape": [512], "dtype": "float16"}],
    "outputs": [{"shape": [512, 512], "dtype": "float16"}],
    "accum_dtype": "float32",
}


def test_doc_example_parses():
    r = CompileRequest.from_json(json.dumps(DOC_REQUEST))
    assert (r.pattern, r.M, r.N, r.K, r.dtype) == ("linear_relu", 512, 512, 256, torch.float16)


@pytest.mark.parametrize("mutate,msg", [
    (lambda r: r.update(ops=["matmul", "add", "gelu"]), "do not form"),
    (lambda r: r.update(pattern="ffn_two_layer", ops=["matmul", "add", "relu", "matmul", "add"]),
     "not a fused GEMM or chain the engine plans"),
    (lambda r: r["inputs"][1].update(shape=[255, 512]), "inner dimensions"),
    (lambda r: r["outputs"][0].update(shape=[512, 511]), "output shape"),
    (lambda r: r["inputs"][2].update(shape=[511]), "bias shape"),
    (lambda r: r["inputs"][0].update(dtype="bfloat16"), "share one of"),
    (lambda r: r.update(accum_dtype="float16"), "float32 accumulation"),
    (lambda r: r.pop("inputs"), "lacks 'inputs'"),
])
def test_request_validation(mutate, msg):
    req = json.loads(json.dumps(DOC_REQUEST))
    mutate(req)
    with pytest.raises(CompileError, match=msg):
        CompileRequest.from_json(req)


def test_attention_score_request_carries_scale():
    req = {"pattern": "attention_score", "ops": ["matmul", "mul"], "scale": 0.125,
           "inputs": [{"shape": [64, 32], "dtype": "bfloat16"},
                      {"shape": [32, 64], "dtype": "bfloat16"},
                      {"shape": [1], "dtype": "bfloat16"}],
           "outputs": [{"shape": [64, 64], "dtype": "bfloat16"}]}
    r = CompileRequest.from_json(req)
    assert r.pattern == "attention_score" and r.scale == 0.125


def test_plan_cache_keys_by_shape():
    _build.build()
    cache = PlanCache()
    p1 = cache.get(DOC_REQUEST)
    p2 = cache.get(json.dumps(DOC_REQUEST))
    assert p1 is p2 and cache.hits == 1 and cache.misses == 1
    other = json.loads(json.dumps(DOC_REQUEST))
    other["inputs"][0]["shape"] = [128, 256]
    other["outputs"][0]["shape"] = [128, 512]
    assert cache.get(other) is not p1 and len(cache) == 2


def test_plan_rejects_wrong_operands_on_cpu():
    _build.build()
    plan = PlanCache().get(DOC_REQUEST)
    with pytest.raises(ValueError, match="x must be"):
        plan(torch.zeros(4, 4, dtype=torch.float16), torch.zeros(256, 512, dtype=torch.float16))


def test_request_round_trips_through_json():
    r = CompileRequest.from_json(DOC_REQUEST)
    assert CompileRequest.from_json(json.dumps(r.to_json())) == r
    other = json.loads(json.dumps(DOC_REQUEST))
    other["inputs"][0]["shape"] = [256, 256]
    other["outputs"][0]["shape"] = [256, 512]
    assert CompileRequest.from_json(other).shape_hash != r.shape_hash


def test_kvspace_backed_cache_records_versions():
    from deepx_op_gpukernelcompiler_b200.kvspace_local import KVSpace
    from deepx_op_gpukernelcompiler_b200.plan import record_key
    _build.build()
    kv = KVSpace()
    first = PlanCache(kv)
    first.get(DOC_REQUEST)
    small = json.loads(json.dumps(DOC_REQUEST))
    small["inputs"][0]["shape"] = [4, 256]
    small["outputs"][0]["shape"] = [4, 512]
    first.get(small)
    assert first.misses == 2 and first.kv_hits == 0
    recs = first.records("__fusion_0")
    assert len(recs) == 2
    req = CompileRequest.from_json(DOC_REQUEST)
    rec = recs[req.shape_hash]
    assert record_key(req) == f"/func/__fusion_0_b200/{req.shape_hash}"
    assert rec["entry"] == "dx_plan_call" and rec["library"] == "libdeepx_fused.so"
    assert rec["kernel"] == "umma" and recs[CompileRequest.from_json(small).shape_hash]["kernel"] == "decode"
    assert CompileRequest.from_json(rec["request"]) == req
    # A second process-level cache over the same store finds the versions.
    second = PlanCache(kv)
    second.get(json.dumps(DOC_REQUEST))
    assert second.kv_hits == 1 and second.misses == 0


def test_kvspace_record_collision_is_rejected():
    from deepx_op_gpukernelcompiler_b200.kvspace_local import KVSpace
    from deepx_op_gpukernelcompiler_b200.plan import record_key
    _build.build()
    kv = KVSpace()
    req = CompileRequest.from_json(DOC_REQUEST)
    bogus = json.loads(json.dumps(DOC_REQUEST))
    bogus["inputs"][0]["shape"] = [64, 256]
    bogus["outputs"][0]["shape"] = [64, 512]
    kv.set(record_key(req), json.dumps({"request": bogus}))
    with pytest.raises(CompileError, match="collision"):
        PlanCache(kv).get(DOC_REQUEST)


def test_plan_cache_is_thread_safe():
    """Concurrent lookups of the same and different requests build each plan
    once and hand every thread the same object."""
    import threading
    _build.build()
    cache = PlanCache()
    reqs = []
    for m in (16, 64, 256, 512):
        r = json.loads(json.dumps(DOC_REQUEST))
        r["inputs"][0]["shape"] = [m, 256]
        r["outputs"][0]["shape"] = [m, 512]
        reqs.append(r)
    got = [[None] * 32 for _ in reqs]

    def worker(t):
        for i, r in enumerate(reqs):
            got[i][t] = cache.get(r)

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(32)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert len(cache) == len(reqs) and cache.misses == len(reqs)
    assert cache.hits == 32 * len(reqs) - len(reqs)
    for row in got:
        assert all(p is row[0] for p in row)


def _mlp_request(M=512, K=256, H=1024, dt="bfloat16"):
    return {"func": "mlp_block", "pattern": "mlp_residual",
            "ops": ["matmul", "add", "gelu", "matmul", "add", "add"],
            "inputs": [{"shape": s, "dtype": dt} for s in ([M, K], [K, H], [H], [H, K], [K])],
            "outputs": [{"shape": [M, K], "dtype": dt}]}


def test_mlp_residual_request_round_trips():
    r = CompileRequest.from_json(_mlp_request())
    assert (r.pattern, r.M, r.N, r.K) == ("mlp_residual", 512, 1024, 256)
    assert CompileRequest.from_json(r.to_json()).key == r.key


@pytest.mark.parametrize("mutate,msg", [
    (lambda r: r["inputs"].pop(), "takes 5 inputs"),
    (lambda r: r["inputs"][3].update(shape=[1024, 128]), "input shapes"),
    (lambda r: r["outputs"][0].update(shape=[512, 1024]), "output shape"),
])
def test_mlp_residual_request_validation(mutate, msg):
    req = _mlp_request()
    mutate(req)
    with pytest.raises(CompileError, match=msg):
        CompileRequest.from_json(req)
