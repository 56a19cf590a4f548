"""Oracle for the negative L1 distance projection (test infrastructure only).

Restates ``negative_l1_distance`` (layers/triton_negative_l1.py:233-241),
whose CPU path is ``-torch.cdist(x, prototype, p=1)`` and whose CUDA path
accumulates ``-sum_f |x[m,f] - w[p,f]|`` in fp32 (:19-52).
"""

from __future__ import annotations

import numpy as np
import torch


def negative_l1_torch(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """The reference's CPU path verbatim in meaning: ``-cdist(x, w, p=1)``."""
    return -torch.cdist(x, w, p=1)


def negative_l1_np(x, w, *, dtype=np.float64, block: int = 256) -> np.ndarray:
    """Blocked numpy restatement with ``dtype`` accumulation."""
    x = np.asarray(x, dtype=dtype)
    w = np.asarray(w, dtype=dtype)
    out = np.empty((x.shape[0], w.shape[0]), dtype=dtype)
    for start in range(0, x.shape[0], block):
        chunk = x[start:start + block]
        out[start:start + block] = -np.abs(chunk[:, None, :] - w[None, :, :]).sum(axis=-1)
    return out
