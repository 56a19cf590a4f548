"""Oracle restatement of the hex-lattice pair geometry (test infrastructure only).

Written with scalar Python loops so it shares no code with the product's
vectorised ``intp_preliminary_b200/hexgrid.py``:
  * axial coordinates, ring distance and six-sector directions follow
    utils/hex_graph.py:15-47 (``xy_to_axial``, ``hex_relative_bins``);
  * the synthetic Look configurations bin a pair by
    ``floor(n_dir * atan2(dy, dx) / 2pi) mod n_dir`` (with a 1e-9 nudge for
    pairs exactly on a bin edge) and hex ring ``1..n_rad``; the slot of a
    pair is ``dir * n_rad + ring - 1`` and ring 0 / ring > n_rad carry none.
"""

from __future__ import annotations

import math

SLOT_NONE = 255


def lattice_points(rows: int, cols: int) -> list[tuple[float, float]]:
    points = []
    for r in range(rows):
        for c in range(cols):
            points.append((c + 0.5 * (r % 2), r * math.sqrt(3.0) / 2.0))
    return points


def axial(point: tuple[float, float]) -> tuple[int, int]:
    x, y = point
    r = round(2.0 * y / math.sqrt(3.0))
    q = round(x - 0.5 * r)
    return int(q), int(r)


def ring(a: tuple[float, float], b: tuple[float, float]) -> int:
    qa, ra = axial(a)
    qb, rb = axial(b)
    dq, dr = qb - qa, rb - ra
    return (abs(dq) + abs(dr) + abs(dq + dr)) // 2


def direction(a, b, n_dir: int) -> int:
    angle = math.atan2(b[1] - a[1], b[0] - a[0])
    return int(math.floor(n_dir * angle / (2.0 * math.pi) + 1e-9)) % n_dir


def six_sector(a, b) -> int:
    if ring(a, b) == 0:
        return 0
    angle = math.atan2(b[1] - a[1], b[0] - a[0])
    return int(math.floor((angle + math.pi / 6.0) / (math.pi / 3.0))) % 6


def slot_table(points, n_dir: int, n_rad: int) -> list[list[int]]:
    table = []
    for a in points:
        row = []
        for b in points:
            rg = ring(a, b)
            row.append(direction(a, b, n_dir) * n_rad + rg - 1 if 1 <= rg <= n_rad else SLOT_NONE)
        table.append(row)
    return table
