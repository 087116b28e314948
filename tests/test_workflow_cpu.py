"""Host-side workflow and harness behaviour that needs no GPU (CPU)."""
from pathlib import Path

import pytest

import deepx_op_gpukernelcompiler_b200 as pkg
from deepx_op_gpukernelcompiler_b200 import compile_and_test, kvload, workflow
from deepx_op_gpukernelcompiler_b200.kvspace_local import KVSpace

KV_DIR = Path(pkg.__file__).parent / "kv"


@pytest.fixture()
def kv():
    store = KVSpace()
    kvload.load_dir(store, KV_DIR, pkg="fusion_cases")
    return store


def test_compile_and_test_reports_non_compilable(kv):
    r = compile_and_test(kv, "/func/fusion_cases/sequential_gelu")
    assert not r.success and r.error == "multi_kernel: ffn_sequential"
    r = compile_and_test(kv, "/func/fusion_cases/masked_softmax")
    assert not r.success and r.error == "needs_template: attention_softmax"


def test_engine_chains_need_a_gpu(kv):
    """ffn_two_layer / ffn_gated run as fused chains: on a CPU-only host the
    call fails loudly instead of falling back."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    for name in ("two_layer_relu", "gated_silu"):
        with pytest.raises(RuntimeError, match="needs a CUDA device"):
            compile_and_test(kv, f"/func/fusion_cases/{name}")


def test_compile_and_test_reports_unmatched():
    store = KVSpace()
    kvload.store_func(store, "x", {"name": "f", "signature": "def f(a) -> (b)",
                                   "ops": [{"op": "tensor.tanh", "reads": ["a"], "writes": ["b"]}]})
    r = compile_and_test(store, "/func/x/f")
    assert r.error == "no fusion pattern for: tensor.tanh"


def test_unknown_engine_is_rejected(capsys):
    with pytest.raises(SystemExit) as ei:
        workflow.main(["--fusion", "tilelang", "--all"])
    assert ei.value.code == 1
    assert "unknown fusion engine" in capsys.readouterr().out


def test_workflow_non_compilable_exits_1(capsys):
    with pytest.raises(SystemExit) as ei:
        workflow.main(["--load", str(KV_DIR), "/func/fusion_cases/two_layer_relu"])
    assert ei.value.code == 1
    out = capsys.readouterr().out
    assert "fuse: ffn_two_layer  status: multi_kernel" in out


def test_workflow_usage(capsys):
    with pytest.raises(SystemExit):
        workflow.main([])
    assert "usage" in capsys.readouterr().out


def test_engine_registry_has_only_the_b200_engine():
    assert list(pkg.ENGINES) == ["b200"]
    assert pkg.ENGINES["b200"] is pkg.make_linear_kernel
