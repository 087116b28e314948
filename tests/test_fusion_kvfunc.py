"""Pattern matching and kvspace IR reading against the reference (CPU).

Golden data: tests/golden/reference_classify.json, produced by the
reference's own ``kvfunc.read_func`` / ``list_funcs`` and ``fusion.classify``
on every reference fixture (test/fusion_cases/*.kv, test/inference.kv).
"""
import pytest

from deepx_op_gpukernelcompiler_b200 import FUSION_DB, classify, fusion, kvload, list_funcs, read_func
from deepx_op_gpukernelcompiler_b200.kvspace_local import ErrNotFound, KVSpace
from golden_data import classify_data

CASES = classify_data()["cases"]


def _store_case(kv, case):
    name = case["path"].rsplit("/", 1)[-1]
    kvload.store_func(kv, case["path"].split("/")[2],
                      {"name": name, "signature": case["signature"], "ops": case["ops"]})


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["file"])
def test_classify_matches_reference(case):
    got = list(classify(case["ops"]))
    assert got == case["classify"]


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["file"])
def test_read_func_matches_reference(case):
    kv = KVSpace()
    _store_case(kv, case)
    f = read_func(kv, case["path"])
    assert f["signature"] == case["signature"]
    assert f["ops"] == case["ops"]


def test_list_funcs_matches_reference():
    kv = KVSpace()
    for c in CASES:
        _store_case(kv, c)
    assert list_funcs(kv, "/func/fusion_cases") == classify_data()["list_funcs"]
    assert list_funcs(kv, "/func/nowhere") == []


def test_reference_rows_are_identical():
    ref = {tuple(r["ops"]): tuple(r["value"]) for r in classify_data()["fusion_db"]}
    assert fusion.REFERENCE_DB == ref
    for key, val in ref.items():
        assert FUSION_DB[key] == val


def test_extension_rows_do_not_shadow_reference():
    ref = {tuple(r["ops"]) for r in classify_data()["fusion_db"]}
    assert not (set(fusion.EXTENSION_DB) & ref)


def test_extension_patterns():
    def ops(*names):
        return [{"op": f"tensor.{n}", "reads": [], "writes": []} for n in names] + \
               [{"op": "return", "reads": [], "writes": []}]
    assert classify(ops("matmul", "add", "add")) == (
        "linear_residual", "linear_residual", None, "compilable")
    assert classify(ops("matmul", "add", "gelu", "matmul", "add", "add")) == (
        "mlp_residual", "mlp_chain", "gelu", "compilable")
    assert classify(ops("matmul", "add", "tanh"))[3] == "not_matched"


def test_kv_loader_parses_comments_and_multiple_functions():
    src = """
    // two functions in one file
    def f(x, W, b) -> (y) {
        tensor.matmul(x, W) -> t   // product
        tensor.add(t, b) -> y
    }
    def g(a) -> (o) {
        tensor.relu(a) -> o
    }
    """
    funcs = kvload.parse_kv(src)
    assert [f["name"] for f in funcs] == ["f", "g"]
    assert funcs[0]["ops"][0] == {"op": "tensor.matmul", "reads": ["x", "W"], "writes": ["t"]}
    kv = KVSpace()
    for f in funcs:
        kvload.store_func(kv, "demo", f)
    assert list_funcs(kv, "/func/demo") == ["f", "g"]
    assert read_func(kv, "/func/demo/g")["ops"] == [
        {"op": "tensor.relu", "reads": ["a"], "writes": ["o"]}]


def test_kv_loader_rejects_garbage():
    with pytest.raises(kvload.KvSyntaxError):
        kvload.parse_kv("def f(x) -> (y) {\n  this is not an op\n}")


def test_kvspace_semantics():
    kv = KVSpace()
    with pytest.raises(ErrNotFound):
        kv.get("/missing")
    with pytest.raises(ErrNotFound):
        kv.list("/missing")
    kv.set("/func/p/f", "sig")
    kv.set("/func/p/f/[0,0]", "tensor.add")
    kv.set("/func/p/meta", 3)
    assert kv.get("/func/p/f").kind == "string"
    assert kv.get("/func/p/meta").kind != "string"
    assert kv.list("/func/p") == ["f", "meta"]
    assert list_funcs(kv, "/func/p") == ["f"]  # non-string children skipped
    with pytest.raises(ErrNotFound):
        read_func(kv, "/func/p/absent")


def test_package_fixtures_classify():
    """The .kv fixtures shipped with the package cover every compilable pattern."""
    from pathlib import Path
    import deepx_op_gpukernelcompiler_b200 as pkg
    kv = KVSpace()
    paths = kvload.load_dir(kv, Path(pkg.__file__).parent / "kv", pkg="fusion_cases")
    patterns = {classify(read_func(kv, p)["ops"])[0] for p in paths}
    assert {"linear", "linear_relu", "linear_gelu", "linear_silu", "linear_swish",
            "linear_residual", "mlp_residual"} <= patterns
