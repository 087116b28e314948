"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run where a checkout of the reference is readable, giving its root as the
argument or in DEEPX_REFERENCE_DIR:

    python tests/golden/make_golden.py /path/to/deepx-op-gpukernelcompiler

What it writes, and from which reference code:

* ``reference_classify.json`` — for every reference fixture
  (test/fusion_cases/*.kv, test/inference.kv): the op list read back by the
  reference's own ``kvfunc.read_func`` (deepx_op_gpukernelcompiler/
  kvfunc.py:13-34) and the result of the reference's ``fusion.classify``
  (fusion.py:95-109); plus ``list_funcs`` (kvfunc.py:37-52) over the loaded
  store and the full ``FUSION_DB`` table (fusion.py:14-85).  The .kv text is
  loaded into an in-memory store by this repo's loader, standing in for the
  external ``kvlang load``.
* ``golden_linear.npz`` + ``golden_cases.json`` — seeded inputs and the
  reference oracle's output for each case: ``ref = a @ b + bias`` then
  ``ACTIVATION_PT[act](ref)`` (kernel.py:64-66, fusion.py:87-92), evaluated
  by torch on CPU in fp32 on the (cast) inputs, with the reference module's
  own ACTIVATION_PT.  The erf-GELU case uses the reference kernels' formula
  0.5*x*(erf(x*0.7071067811865475)+1) (kernel_triton.py:61).  Residual
  cases add R after the activation; the MLP case chains two such calls.
  Gated cases follow the ``ffn_gated`` chain op by op
  (test/fusion_cases/07_ffn_gated.kv): the gate through the same expression
  with ``ACTIVATION_PT['silu']``, the up projection without activation, their
  product (tensor.mul), and for the full chain one more linear.

Inputs: torch.Generator(seed), X ~ N(0,1), W ~ N(0, 1/K), bias ~ U(-0.1, 0.1),
generated in fp32 and cast to the case dtype.  Inputs are stored in their
own width (bf16 as uint16 bit patterns); outputs Y as float32.
"""
from __future__ import annotations

import importlib.util
import json
import math
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from deepx_op_gpukernelcompiler_b200 import kvload, kvspace_local  # noqa: E402

DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _import_reference(ref_root: Path):
    """Import the reference's fusion.py and kvfunc.py by path.

    kvfunc.py imports the external ``kvspace`` client, which is not
    installed; this repo's dict-backed stand-in is registered under that
    name first.
    """
    shim = types.ModuleType("kvspace")
    shim.KVSpace = kvspace_local.KVSpace
    shim.ErrNotFound = kvspace_local.ErrNotFound
    shim.connect = lambda: kvspace_local.KVSpace()
    sys.modules.setdefault("kvspace", shim)
    pkg = ref_root / "deepx_op_gpukernelcompiler"
    mods = {}
    for name in ("fusion", "kvfunc"):
        spec = importlib.util.spec_from_file_location(f"_ref_{name}", pkg / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods["fusion"], mods["kvfunc"]


def make_classify(ref_root: Path, fusion, kvfunc) -> dict:
    kv = kvspace_local.KVSpace()
    files = sorted((ref_root / "test" / "fusion_cases").glob("*.kv")) + [ref_root / "test" / "inference.kv"]
    cases = []
    for f in files:
        pkg = "fusion_cases" if f.parent.name == "fusion_cases" else "test"
        for path in kvload.load_file(kv, f, pkg=pkg):
            func = kvfunc.read_func(kv, path)
            pattern, template, activation, status = fusion.classify(func["ops"])
            cases.append({
                "file": f"{f.parent.name}/{f.name}",
                "path": path,
                "signature": func["signature"],
                "ops": func["ops"],
                "classify": [pattern, template, activation, status],
            })
    db = [{"ops": list(k), "value": list(v)} for k, v in fusion.FUSION_DB.items()]
    return {
        "cases": cases,
        "list_funcs": kvfunc.list_funcs(kv, "/func/fusion_cases"),
        "fusion_db": db,
    }


def _gen(seed, M, K, N, dtype, residual=False):
    g = torch.Generator().manual_seed(seed)
    dt = DTYPES[dtype]
    X = torch.randn(M, K, generator=g).to(dt)
    W = (torch.randn(K, N, generator=g) / math.sqrt(K)).to(dt)
    b = (torch.rand(N, generator=g) * 0.2 - 0.1).to(dt)
    R = torch.randn(M, N, generator=g).to(dt) if residual else None
    return X, W, b, R


def _store(t: torch.Tensor) -> np.ndarray:
    """Inputs are kept in their own width: fp32 as float32, fp16 as float16,
    bf16 as the uint16 bit pattern (numpy has no bfloat16)."""
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.numpy()
    return t.float().numpy()


def _reference_expr(fusion, a, b, bias, act, R=None):
    """kernel.py:64-66 in fp32 on CPU (+ residual after the activation)."""
    ref = a.float() @ b.float() + bias.float()
    if act == "gelu_erf":
        ref = 0.5 * ref * (torch.erf(ref * 0.7071067811865475) + 1.0)
    elif act and act in fusion.ACTIVATION_PT:
        ref = fusion.ACTIVATION_PT[act](ref)
    if R is not None:
        ref = ref + R.float()
    return ref


def make_numeric(fusion) -> tuple[dict, dict]:
    torch.set_num_threads(1)  # deterministic summation order for the fixture
    arrays: dict[str, np.ndarray] = {}
    cases = []

    def add(name, seed, M, K, N, dtype, act, residual=False, mlp_hidden=None):
        if mlp_hidden is None:
            X, W, b, R = _gen(seed, M, K, N, dtype, residual)
            Y = _reference_expr(fusion, X, W, b, act, R)
            tensors = {"X": X, "W": W, "bias": b, "Y": Y}
            if R is not None:
                tensors["R"] = R
        else:
            g = torch.Generator().manual_seed(seed)
            dt = DTYPES[dtype]
            H_ = mlp_hidden
            X = torch.randn(M, K, generator=g).to(dt)
            W1 = (torch.randn(K, H_, generator=g) / math.sqrt(K)).to(dt)
            b1 = (torch.rand(H_, generator=g) * 0.2 - 0.1).to(dt)
            W2 = (torch.randn(H_, K, generator=g) / math.sqrt(H_)).to(dt)
            b2 = (torch.rand(K, generator=g) * 0.2 - 0.1).to(dt)
            H = _reference_expr(fusion, X, W1, b1, act)
            Y = _reference_expr(fusion, H, W2, b2, None, X)
            tensors = {"X": X, "W1": W1, "b1": b1, "W2": W2, "b2": b2, "Y": Y}
        for k, v in tensors.items():
            arrays[f"{name}/{k}"] = _store(v) if k != "Y" else v.float().numpy()
        cases.append({"name": name, "seed": seed, "M": M, "K": K,
                      "N": N if mlp_hidden is None else mlp_hidden,
                      "dtype": dtype, "act": act, "residual": residual,
                      "mlp": mlp_hidden is not None})

    def add_gated(name, seed, M, K, N, dtype, act="silu", ffn=False):
        g = torch.Generator().manual_seed(seed)
        dt = DTYPES[dtype]
        X = torch.randn(M, K, generator=g).to(dt)
        Wg = (torch.randn(K, N, generator=g) / math.sqrt(K)).to(dt)
        bg = (torch.rand(N, generator=g) * 0.2 - 0.1).to(dt)
        Wu = (torch.randn(K, N, generator=g) / math.sqrt(K)).to(dt)
        bu = (torch.rand(N, generator=g) * 0.2 - 0.1).to(dt)
        H = _reference_expr(fusion, X, Wg, bg, act) * _reference_expr(fusion, X, Wu, bu, None)
        tensors = {"X": X, "Wg": Wg, "bg": bg, "Wu": Wu, "bu": bu}
        if ffn:
            Wo = (torch.randn(N, K, generator=g) / math.sqrt(N)).to(dt)
            bo = (torch.rand(K, generator=g) * 0.2 - 0.1).to(dt)
            tensors.update({"Wo": Wo, "bo": bo})
            H = _reference_expr(fusion, H, Wo, bo, None)
        tensors["Y"] = H
        for k, v in tensors.items():
            arrays[f"{name}/{k}"] = _store(v) if k != "Y" else v.float().numpy()
        cases.append({"name": name, "seed": seed, "M": M, "K": K, "N": N, "dtype": dtype,
                      "act": act, "residual": False, "mlp": False, "gated": True, "ffn": ffn})

    # The reference's CPU-runnable configuration: ReLU(X[256,512] W[512,512] + b), fp32, seed 0.
    add("linear_relu_256x512x512_f32", 0, 256, 512, 512, "f32", "relu")
    # Every compilable activation (fusion.py:16-20) in each dtype, ragged sizes.
    seed = 100
    for dtype in ("f32", "f16", "bf16"):
        for act in (None, "relu", "gelu", "silu", "swish", "gelu_erf"):
            add(f"{act or 'none'}_37x80x72_{dtype}", seed, 37, 80, 72, dtype, act)
            seed += 1
    # Tile-boundary shapes for the tensor-core kernels.
    add("gelu_300x192x400_bf16", 201, 300, 192, 400, "bf16", "gelu")
    add("silu_129x520x264_f16", 202, 129, 520, 264, "f16", "silu")
    # Decode-shaped (skinny M) cases.
    add("gelu_erf_16x320x384_f16", 203, 16, 320, 384, "f16", "gelu_erf")
    add("relu_5x384x256_bf16", 204, 5, 384, 256, "bf16", "relu")
    add("silu_40x256x256_bf16", 205, 40, 256, 256, "bf16", "silu")
    # linear_residual: Y = X W + b + R.
    add("residual_96x128x160_bf16", 206, 96, 128, 160, "bf16", None, residual=True)
    add("residual_8x256x192_f16", 207, 8, 256, 192, "f16", None, residual=True)
    # mlp_residual: Y = GELU(X W1 + b1) W2 + b2 + X.
    add("mlp_64x128x256_bf16", 208, 64, 128, None, "bf16", "gelu", mlp_hidden=256)
    # Gated dual GEMM act(X Wg + bg) * (X Wu + bu) and the full ffn_gated chain.
    add_gated("gated_silu_37x80x72_f32", 209, 37, 80, 72, "f32")
    add_gated("gated_silu_16x192x320_f16", 210, 16, 192, 320, "f16")
    add_gated("gated_silu_130x256x200_bf16", 211, 130, 256, 200, "bf16")
    add_gated("gated_silu_300x128x264_bf16", 212, 300, 128, 264, "bf16")
    add_gated("ffn_gated_64x128x256_bf16", 213, 64, 128, 256, "bf16", ffn=True)
    return arrays, {"cases": cases}


def main() -> None:
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DEEPX_REFERENCE_DIR")
    if not arg:
        raise SystemExit("usage: make_golden.py <reference checkout root> "
                         "(or set DEEPX_REFERENCE_DIR)")
    ref_root = Path(arg)
    fusion, kvfunc = _import_reference(ref_root)
    (HERE / "reference_classify.json").write_text(
        json.dumps(make_classify(ref_root, fusion, kvfunc), indent=1, ensure_ascii=False) + "\n")
    arrays, meta = make_numeric(fusion)
    np.savez_compressed(HERE / "golden_linear.npz", **arrays)
    (HERE / "golden_cases.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote {len(meta['cases'])} numeric cases, "
          f"{sum(a.nbytes for a in arrays.values()) / 1e6:.2f} MB raw")


if __name__ == "__main__":
    main()
