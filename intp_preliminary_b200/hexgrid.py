"""Hex-lattice geometry and Look slot tables (host-side, CPU, float64).

This module builds the per-pair index tables the Look-attention kernels read:
for every ordered patch pair (query q, key k) a slot index into the query's
Look field, or ``SLOT_NONE`` when the pair carries no Look bias.

Geometry conventions follow the reference:
  * axial coordinates of a triangular-lattice point: ``r = round(2y/sqrt(3))``,
    ``q = round(x - r/2)`` (utils/hex_graph.py:15-22, ``xy_to_axial``);
  * hex ring distance ``(|dq| + |dr| + |dq+dr|) / 2`` (utils/hex_graph.py:41);
  * six-sector direction ``floor((angle + pi/6) / (pi/3)) mod 6`` with the
    self pair at ring 0 / direction 0 (utils/hex_graph.py:43-46).

The synthetic Look configurations (one CLS token plus an R x C offset-row
lattice, odd rows shifted half a step) bin a pair by direction
``floor(n_dir * atan2(dy, dx) / 2pi) mod n_dir`` and ring ``1..n_rad``; pairs
at ring 0 or beyond ``n_rad`` get no bias.  Angles are evaluated in float64
with a 1e-9 bin-width nudge so pairs that sit exactly on a bin edge (lattice
directions are multiples of 30 degrees) land in the upper bin on every host.
"""

from __future__ import annotations

import math

import numpy as np

SLOT_NONE = 255
_EDGE_NUDGE = 1e-9


def offset_row_lattice(rows: int, cols: int) -> np.ndarray:
    """Patch centres ``(rows*cols, 2)`` of an offset-row hex lattice, unit spacing."""
    if rows < 1 or cols < 1:
        raise ValueError("rows and cols must be positive")
    r, c = np.meshgrid(np.arange(rows, dtype=np.float64), np.arange(cols, dtype=np.float64), indexing="ij")
    x = c + 0.5 * np.mod(r, 2.0)
    y = r * (math.sqrt(3.0) / 2.0)
    return np.stack((x.reshape(-1), y.reshape(-1)), axis=-1)


def xy_to_axial(coordinates: np.ndarray) -> np.ndarray:
    """Triangular-lattice xy -> integer axial ``(q, r)`` (utils/hex_graph.py:15-22)."""
    coordinates = np.asarray(coordinates, dtype=np.float64)
    if coordinates.shape[-1] != 2:
        raise ValueError("coordinates must have shape (..., 2)")
    x, y = coordinates[..., 0], coordinates[..., 1]
    axial_r = np.round(2.0 * y / math.sqrt(3.0))
    axial_q = np.round(x - 0.5 * axial_r)
    return np.stack((axial_q, axial_r), axis=-1).astype(np.int64)


def hex_rings(coordinates: np.ndarray) -> np.ndarray:
    """Ring distance for every ``query -> key`` pair, ``(N, N)`` int64."""
    axial = xy_to_axial(coordinates)
    delta = axial[None, :, :] - axial[:, None, :]
    dq, dr = delta[..., 0], delta[..., 1]
    return (np.abs(dq) + np.abs(dr) + np.abs(dq + dr)) // 2


def pair_angles(coordinates: np.ndarray) -> np.ndarray:
    """``atan2(dy, dx)`` of ``key - query`` for every pair, float64 ``(N, N)``."""
    coordinates = np.asarray(coordinates, dtype=np.float64)
    delta = coordinates[None, :, :] - coordinates[:, None, :]
    return np.arctan2(delta[..., 1], delta[..., 0])


def hex_relative_bins(coordinates: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Ring and six-sector direction of every pair (utils/hex_graph.py:25-47)."""
    rings = hex_rings(coordinates)
    angles = pair_angles(coordinates)
    directions = np.mod(np.floor((angles + math.pi / 6.0) / (math.pi / 3.0)).astype(np.int64), 6)
    directions = np.where(rings == 0, 0, directions)
    return rings, directions


def direction_bins(coordinates: np.ndarray, n_dir: int) -> np.ndarray:
    """``floor(n_dir * atan2(dy,dx) / 2pi) mod n_dir`` per pair, int64 ``(N, N)``."""
    if n_dir < 1:
        raise ValueError("n_dir must be positive")
    angles = pair_angles(coordinates)
    position = n_dir * angles / (2.0 * math.pi) + _EDGE_NUDGE
    return np.mod(np.floor(position).astype(np.int64), n_dir)


def direction_radius_slots(coordinates: np.ndarray, n_dir: int, n_rad: int) -> np.ndarray:
    """Slot ``dir * n_rad + (ring - 1)`` for rings ``1..n_rad``, else SLOT_NONE.

    The slot order matches a Look field stored as ``(n_dir, n_rad)`` and
    flattened, i.e. ``pose[..., dir * n_rad + rad - 1]``.
    """
    if n_rad < 1 or n_dir * n_rad > 254:
        raise ValueError("need 1 <= n_rad and n_dir * n_rad <= 254")
    rings = hex_rings(coordinates)
    dirs = direction_bins(coordinates, n_dir)
    valid = (rings >= 1) & (rings <= n_rad)
    slots = np.where(valid, dirs * n_rad + (rings - 1), SLOT_NONE)
    return slots.astype(np.uint8)


def synthetic_look_slots(rows: int, cols: int, n_dir: int, n_rad: int) -> np.ndarray:
    """Slot table of the synthetic ``rows x cols`` offset-row Look configuration."""
    return direction_radius_slots(offset_row_lattice(rows, cols), n_dir, n_rad)
