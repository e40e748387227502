"""Loading helpers for the golden fixtures in ``tests/golden`` (made by make_golden.py)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict:
    with np.load(GOLDEN / name) as data:
        return {k: data[k] for k in data.files}


def known_answers() -> dict:
    return json.loads((GOLDEN / "known_answers.json").read_text())


def to_torch(array, dtype=None, device="cpu"):
    """uint16 arrays become BF16 tensors (bit patterns); others keep their dtype."""
    import torch

    if array.dtype == np.uint16:
        t = torch.from_numpy(array.view(np.int16).copy()).view(torch.bfloat16)
    else:
        t = torch.from_numpy(np.ascontiguousarray(array).copy())
    if dtype is not None:
        t = t.to(dtype)
    return t.to(device)


def bf16_bits(tensor) -> np.ndarray:
    import torch

    return tensor.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def rel_l2(actual, expected) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    return float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))
