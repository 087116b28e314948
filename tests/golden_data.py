"""Access to the committed golden fixtures (tests/golden/)."""
from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


@lru_cache(maxsize=1)
def _npz():
    return dict(np.load(GOLDEN / "golden_linear.npz"))


@lru_cache(maxsize=1)
def cases() -> list[dict]:
    return json.loads((GOLDEN / "golden_cases.json").read_text())["cases"]


@lru_cache(maxsize=1)
def classify_data() -> dict:
    return json.loads((GOLDEN / "reference_classify.json").read_text())


def _tensor(arr: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "bf16":
        return torch.from_numpy(arr.astype(np.uint16).view(np.int16).copy()).view(torch.bfloat16)
    if dtype == "f16":
        return torch.from_numpy(arr.astype(np.float16).copy())
    return torch.from_numpy(arr.astype(np.float32).copy())


def load(case: dict) -> dict[str, torch.Tensor]:
    """Inputs in the case dtype (CPU tensors) and the golden output Y (fp32)."""
    data = _npz()
    prefix = case["name"] + "/"
    out = {}
    for key, arr in data.items():
        if key.startswith(prefix):
            name = key[len(prefix):]
            out[name] = (torch.from_numpy(arr.copy()) if name == "Y"
                         else _tensor(arr, case["dtype"]))
    return out
