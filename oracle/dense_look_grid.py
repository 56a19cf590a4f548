"""Oracle for dense Look-grid sampling (test infrastructure only).

Restates ``reference_dense_look_grid_sample`` (layers/triton_dense_look_grid.py:19-49):
each query's 4 x 12 grid ``grid[b, q, h]`` is sampled at the four corners
(radial0, angular0), (radial0, angular1), (radial1, angular0), (radial1,
angular1) of every key with the bilinear weights (1-rw)(1-aw), (1-rw)aw,
rw(1-aw), rw aw, times valid[q, k]; and its gradient, the scatter-add of
``_DenseLookGridSample.backward`` (:152-181).  The sampling tables are
restated from layers/two_ring_circular_look.py:124-152 for lattices without
reference tables at hand.
"""

from __future__ import annotations

import math

import numpy as np
import torch

TABLE_NAMES = ("radial0", "radial1", "angular0", "angular1", "radial_fraction", "angular_fraction", "valid")


def sampling_tables_np(coordinates) -> dict[str, np.ndarray]:
    """The seven (Q, Q) tables for unit-spaced lattice coordinates (Q, 2).  The
    distance and angle use torch's float32 ``norm`` / ``atan2`` as the reference
    does: at exact lattice distances (d = 2, 3, ...) its rounding decides the
    radial bin, so a different square root would move pairs across bins."""
    xy = torch.as_tensor(np.asarray(coordinates), dtype=torch.float32)
    rel = xy.unsqueeze(0) - xy.unsqueeze(1)
    distance = rel.norm(dim=-1).numpy()
    angle = torch.remainder(torch.atan2(rel[..., 1], rel[..., 0]), 2.0 * math.pi).numpy()
    radial = distance - np.float32(1.0)
    radial0 = np.clip(np.floor(radial), 0, 3).astype(np.int64)
    angular = (angle / np.float32(2 * math.pi) * np.float32(12.0)).astype(np.float32)
    angular0 = np.floor(angular).astype(np.int64) % 12
    return {
        "radial0": radial0,
        "radial1": np.minimum(radial0 + 1, 3),
        "angular0": angular0,
        "angular1": (angular0 + 1) % 12,
        "radial_fraction": np.clip(radial - np.floor(radial), 0.0, 1.0).astype(np.float32),
        "angular_fraction": (angular - np.floor(angular)).astype(np.float32),
        "valid": (distance > 0) & (distance <= 4.0),
    }


def _corners(tables):
    rw = np.asarray(tables["radial_fraction"], dtype=np.float64)
    aw = np.asarray(tables["angular_fraction"], dtype=np.float64)
    r0, r1 = np.asarray(tables["radial0"]), np.asarray(tables["radial1"])
    a0, a1 = np.asarray(tables["angular0"]), np.asarray(tables["angular1"])
    return (((r0, a0), (1 - rw) * (1 - aw)), ((r0, a1), (1 - rw) * aw),
            ((r1, a0), rw * (1 - aw)), ((r1, a1), rw * aw))


def dense_look_grid_np(grid, tables) -> np.ndarray:
    """grid (B, Q, H, 4, 12) -> bias (B, H, Q, Q), float64."""
    g = np.asarray(grid, dtype=np.float64).transpose(0, 2, 1, 3, 4)  # B, H, Q, 4, 12
    batch, heads, queries = g.shape[:3]
    flat = g.reshape(batch, heads, queries, 48)
    valid = np.asarray(tables["valid"]).astype(np.float64)
    qi = np.arange(queries)[:, None]
    out = np.zeros((batch, heads, queries, queries))
    for (r, a), w in _corners(tables):
        out += flat[:, :, qi, r * 12 + a] * w
    return out * valid


def dense_look_grid_grad_np(grad_out, tables) -> np.ndarray:
    """d(sum grad_out * bias)/d grid: (B, Q, H, 4, 12), float64."""
    go = np.asarray(grad_out, dtype=np.float64)  # B, H, Q, K
    batch, heads, queries = go.shape[:3]
    valid = np.asarray(tables["valid"]).astype(np.float64)
    grad = np.zeros((batch, heads, queries, 48))
    qi = np.broadcast_to(np.arange(queries)[:, None], (queries, queries))
    for (r, a), w in _corners(tables):
        contrib = go * (w * valid)
        cell = np.broadcast_to(r * 12 + a, (queries, queries))
        for b in range(batch):
            for h in range(heads):
                np.add.at(grad[b, h], (qi, cell), contrib[b, h])
    return grad.reshape(batch, heads, queries, 4, 12).transpose(0, 2, 1, 3, 4)
