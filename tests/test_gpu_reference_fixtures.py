"""compile_and_test on the reference's own fixture functions (gpu).

The reference drives its engines through ``compile_and_test`` (kernel.py:30-93)
over the functions of ``test/fusion_cases/01..30_*.kv`` and
``test/inference.kv``; this package's ``compile_and_test`` keeps that contract
(CompileResult(success, diff, tl_ms, pt_ms, error), fp16 random inputs,
``diff < 0.5``) with ``ENGINES["b200"]``.  The fixtures are not copied here:
``tests/golden/reference_classify.json`` holds, for each, the op list that the
reference's own ``read_func`` returned when ``tests/golden/make_golden.py``
imported it.  This test writes those op lists into an in-memory store at the
reference's paths and checks, on the GPU:

* every function the reference marks ``compilable`` (01-05 and inference) runs
  with success=True on the engine, and its output matches the PyTorch
  expression the harness compares against (kernel.py:64-66) — the six
  functions the reference itself can compile;
* the chains the engine runs beyond the reference (the two-layer and gated
  FFNs, the attention GEMM templates) succeed too;
* every other function fails the way the reference's harness fails it
  (``"<status>: <pattern>"``, kernel.py:45-46) without launching anything;
* the workflow's ``--all`` summary over the store counts them as the
  reference classifies them.
"""
import json
from pathlib import Path

import pytest

from deepx_op_gpukernelcompiler_b200 import compile_and_test, workflow
from deepx_op_gpukernelcompiler_b200.kvload import store_func
from deepx_op_gpukernelcompiler_b200.kvspace_local import KVSpace

pytestmark = pytest.mark.gpu

FIXTURES = json.loads((Path(__file__).parent / "golden" / "reference_classify.json").read_text())
CASES = {c["path"]: c for c in FIXTURES["cases"]}
COMPILABLE = sorted(p for p, c in CASES.items() if c["classify"][3] == "compilable")
ENGINE_EXTRA = {"ffn_two_layer", "ffn_gated", "attention_output", "attention_score"}


@pytest.fixture(scope="module")
def kv():
    store = KVSpace()
    for path, case in CASES.items():
        pkg, name = path.split("/")[2], path.split("/")[3]
        got = store_func(store, pkg, {"name": name, "signature": case["signature"],
                                      "ops": case["ops"]})
        assert got == path
    return store


def test_reference_compilable_set():
    names = {CASES[p]["classify"][0] for p in COMPILABLE}
    assert names == {"linear", "linear_relu", "linear_gelu", "linear_silu", "linear_swish"}
    assert len(COMPILABLE) == 6  # 01-05 and test/inference.kv


@pytest.mark.parametrize("path", COMPILABLE)
@pytest.mark.parametrize("seed", [0, 1])
def test_reference_compilable_functions_run_on_the_engine(kv, path, seed):
    r = compile_and_test(kv, path, seed=seed, n_iter=5, warmup=2)
    assert r.error is None and r.success, (path, r)
    # fp16 inputs N(0,1), K=256: the harness's own pass mark is diff < 0.5;
    # the fused fp32-accumulate kernel stays within half of it.
    assert r.diff < 0.25, (path, r.diff)
    assert r.tl_ms > 0 and r.pt_ms > 0


@pytest.mark.parametrize("path", sorted(p for p, c in CASES.items()
                                        if c["classify"][0] in ENGINE_EXTRA))
def test_engine_chains_beyond_the_reference(kv, path):
    r = compile_and_test(kv, path, seed=0, n_iter=3, warmup=1)
    assert r.error is None and r.success, (path, r)


@pytest.mark.parametrize("path", sorted(p for p, c in CASES.items()
                                        if c["classify"][3] != "compilable"
                                        and c["classify"][0] not in ENGINE_EXTRA))
def test_other_functions_fail_like_the_reference(kv, path):
    pattern, _, _, status = CASES[path]["classify"]
    r = compile_and_test(kv, path, seed=0, n_iter=1, warmup=0)
    assert not r.success
    assert r.error == f"{status}: {pattern}", (path, r.error)


def test_workflow_summary_over_reference_functions(kv, capsys):
    workflow._run_all(kv, "b200", "/func/fusion_cases")
    out = capsys.readouterr().out
    n_comp = sum(1 for p, c in CASES.items()
                 if p.startswith("/func/fusion_cases/") and c["classify"][3] == "compilable")
    assert "summary" in out and f"compilable: {n_comp}" in out
