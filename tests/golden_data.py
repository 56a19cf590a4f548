"""Loaders for the golden fixtures (generated from the reference by make_golden.py)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / name) as data:
        return {key: data[key] for key in data.files}


def tensor(array: np.ndarray, dtype: torch.dtype | None = None) -> torch.Tensor:
    """int16 arrays hold bf16 bit patterns; everything else is taken as is."""
    if array.dtype == np.int16:
        t = torch.from_numpy(array.copy()).view(torch.bfloat16)
    else:
        t = torch.from_numpy(array.copy())
    return t if dtype is None else t.to(dtype)
