"""The reference's own harness, unmodified, driving this engine.

Switching the reference over to this engine is one added entry in its
``ENGINES`` table (kernel.py:14-17): ``"b200": make_linear_kernel``.  This
test does exactly that to the reference package installed (unmodified, by
pip) under ``baseline/_ref`` — or under ``$DEEPX_REFERENCE_PKG`` — and then
runs the reference's own code:

* ``compile_and_test(kv, path, fusion="b200")`` (kernel.py:30-93) on the six
  functions it classifies as compilable (test/fusion_cases/01-05 and
  test/inference.kv): its fp16 inputs, its ``diff < 0.5`` mark, its 20 + 200
  launch timing;
* the same call on every other fixture function, which the harness must
  refuse with its own error before any launch (these two checks, and the
  read-back of the stored functions, need no GPU);
* ``workflow._run_all(kv, "b200")`` (workflow.py:79-111), its summary table
  over /func/fusion_cases.

The fixture functions come from ``tests/golden/reference_classify.json`` (the
op lists the reference's own ``read_func`` returned), stored at the
reference's paths in this package's in-process KVSpace.  The reference
imports a ``kvspace`` client (kvspace-py) that this image lacks; this
package's KVSpace has the surface the reference uses (``get`` → value with
``kind``/``as_str``, ``list``, ``ErrNotFound``, ``connect``) and stands in for
it.  Skipped when the reference package is not installed.
"""
import importlib
import importlib.util
import json
import os
import sys
from pathlib import Path

import pytest

from deepx_op_gpukernelcompiler_b200 import kvspace_local
from deepx_op_gpukernelcompiler_b200.kernel_b200 import make_linear_kernel
from deepx_op_gpukernelcompiler_b200.kvload import store_func

ROOT = Path(__file__).resolve().parent.parent
REF = Path(os.environ.get("DEEPX_REFERENCE_PKG", ROOT / "baseline" / "_ref"))
FIXTURES = json.loads((Path(__file__).parent / "golden" / "reference_classify.json").read_text())
CASES = {c["path"]: c for c in FIXTURES["cases"]}
COMPILABLE = sorted(p for p, c in CASES.items() if c["classify"][3] == "compilable")

pytestmark = pytest.mark.skipif(not (REF / "deepx_op_gpukernelcompiler" / "kernel.py").exists(),
                                reason=f"reference package not installed under {REF}")


@pytest.fixture(scope="module")
def ref():
    added_kvspace = importlib.util.find_spec("kvspace") is None
    if added_kvspace:
        sys.modules["kvspace"] = kvspace_local
    sys.path.insert(0, str(REF))
    try:
        kernel = importlib.import_module("deepx_op_gpukernelcompiler.kernel")
        workflow = importlib.import_module("deepx_op_gpukernelcompiler.workflow")
        assert Path(kernel.__file__).resolve().is_relative_to(REF.resolve()), kernel.__file__
        kernel.ENGINES["b200"] = make_linear_kernel  # the one-line switch-over
        yield kernel, workflow
    finally:
        sys.path.remove(str(REF))
        for name in [m for m in sys.modules if m == "deepx_op_gpukernelcompiler"
                     or m.startswith("deepx_op_gpukernelcompiler.")]:
            del sys.modules[name]
        if added_kvspace:
            del sys.modules["kvspace"]


@pytest.fixture(scope="module")
def kv():
    store = kvspace_local.KVSpace()
    for path, case in CASES.items():
        pkg, name = path.split("/")[2], path.split("/")[3]
        assert store_func(store, pkg, {"name": name, "signature": case["signature"],
                                       "ops": case["ops"]}) == path
    return store


def test_reference_reads_the_stored_functions(ref, kv):
    kernel, _ = ref
    read_func = importlib.import_module("deepx_op_gpukernelcompiler.kvfunc").read_func
    for path, case in CASES.items():
        assert read_func(kv, path)["ops"] == case["ops"], path


@pytest.mark.gpu
@pytest.mark.parametrize("path", COMPILABLE)
def test_reference_compile_and_test_on_this_engine(ref, kv, path):
    kernel, _ = ref
    r = kernel.compile_and_test(kv, path, fusion="b200")
    assert r.error is None, (path, r.error)
    assert r.success and r.diff < 0.5, (path, r.diff)
    assert r.tl_ms > 0 and r.pt_ms > 0
    print(f"{path}: diff {r.diff:.4f}  b200 {r.tl_ms:.4f} ms  PyTorch {r.pt_ms:.4f} ms")


@pytest.mark.parametrize("path", sorted(p for p, c in CASES.items()
                                        if c["classify"][3] != "compilable"))
def test_reference_refuses_the_rest(ref, kv, path):
    kernel, _ = ref
    pattern, _, _, status = CASES[path]["classify"]
    r = kernel.compile_and_test(kv, path, fusion="b200")  # returns before any launch
    assert not r.success
    if status == "not_matched":  # the harness names the op sequence (kernel.py:42-44)
        ops = " → ".join(o["op"] for o in CASES[path]["ops"] if o["op"] != "return")
        want = f"no fusion pattern for: {ops}"
    else:
        want = f"{status}: {pattern}"
    assert r.error == want, (path, r.error)


@pytest.mark.gpu
def test_reference_workflow_summary(ref, kv, capsys):
    _, workflow = ref
    workflow._run_all(kv, "b200")
    out = capsys.readouterr().out
    n_comp = sum(1 for p, c in CASES.items()
                 if p.startswith("/func/fusion_cases/") and c["classify"][3] == "compilable")
    assert "engine: b200" in out and "summary" in out
    assert f"compilable: {n_comp}" in out, out
    assert "❌" not in out
