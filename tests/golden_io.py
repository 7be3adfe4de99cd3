"""Loader for the golden vectors written by tests/golden/make_golden.py."""
from __future__ import annotations

from functools import lru_cache
from pathlib import Path

import numpy as np
import torch

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"


@lru_cache(maxsize=None)
def load(name: str) -> dict[str, dict[str, torch.Tensor]]:
    """{case: {key: tensor or str}}; bf16 tensors are restored from their bit patterns."""
    data = np.load(GOLDEN_DIR / f"{name}.npz")
    cases: dict[str, dict[str, torch.Tensor]] = {}
    for full in data.files:
        case, key = full.split("/", 1)
        arr = data[full]
        if key.endswith("__bf16"):
            t = torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
            key = key[: -len("__bf16")]
        elif arr.dtype.kind == "U":          # strings (e.g. a recorded error message)
            t = str(arr)
        else:
            t = torch.from_numpy(np.array(arr))
        cases.setdefault(case, {})[key] = t
    return cases
