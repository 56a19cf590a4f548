"""Slot grouping of the Look fields' pair geometry (CPU).

The compact SLOT_FIELDS form replaces the reference's dense (36, 12, 195, 195)
Look fields by per-slot values gathered through a pair table.  These tests
bound the error of that grouping: against the product's own table builder
(``share_vit.look_slot_basis``) and, when the reference is installed in
baseline/_ref, against the fields the reference's ``SquarePatchDenseGridLook``
itself computes (layers/square_patch_dense_grid_look.py:357-379).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from intp_preliminary_b200.look_registry import group_pairs, pair_weights_from_tables
from intp_preliminary_b200.share_vit import HexSupport, look_sampling_tables, look_slot_basis

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


def _product_tables():
    """The product's restated sampling tables as the seven named (12, Np, Np) buffers."""
    unit_xy = HexSupport(24).unit_xy
    index, weight = look_sampling_tables(unit_xy)
    return unit_xy, index, weight


def test_grouping_matches_look_slot_basis_partition():
    unit_xy, index, weight = _product_tables()
    table, basis = look_slot_basis(unit_xy)
    planes, n = index.shape[:2]
    dense = torch.zeros(planes, n, n, 48, dtype=torch.float64)
    dense.scatter_add_(-1, index, weight.double())
    weights = dense.permute(1, 2, 0, 3).reshape(n * n, planes, 48).numpy()
    flat, representative, error = group_pairs(weights)
    assert representative.size == basis.shape[-1] == 68
    # the same partition of the pairs (slot numbers may differ)
    a, b = table.reshape(-1).astype(np.int64), flat.astype(np.int64)
    assert ((a == 255) == (b == 255)).all()
    pairs = np.stack([a[a != 255], b[b != 255]], axis=1)
    assert np.unique(pairs, axis=0).shape[0] == 68
    # pairs merged into one slot differ only by float32 noise in their weights
    assert error <= 1e-5


def test_group_pairs_keeps_distinct_geometry_apart():
    w = np.zeros((5, 2, 3))
    w[0, 0, 0] = 1.0
    w[1, 0, 0] = 1.0 + 3e-7      # float noise: merged with pair 0
    w[2, 0, 0] = 0.5             # different weight: own slot
    w[3, 1, 2] = 1.0             # different plane / cell: own slot
    table, representative, error = group_pairs(w)
    assert table.tolist() == [0, 0, 1, 2, 255]
    assert representative.tolist() == [0, 2, 3]
    assert error == pytest.approx(3e-7)


@pytest.mark.skipif(not (REF / "layers" / "square_patch_dense_grid_look.py").exists(),
                    reason="reference not installed in baseline/_ref")
def test_slot_values_reproduce_reference_fields():
    """Per-slot values gathered from the reference's own fields at each slot's
    first pair reproduce every field value within weight_error * max|grid|."""
    sys.path.insert(0, str(REF))
    saved = {k: v for k, v in sys.modules.items() if k.split(".")[0] in ("layers", "model", "utils")}
    for key in saved:
        del sys.modules[key]
    try:
        from layers.square_patch_dense_grid_look import SquarePatchDenseGridLook
        from model.deit_tiny_rot_hex_look import DeiTTinyRotHexLook

        from intp_preliminary_b200.look_registry import slot_geometry_of

        model = DeiTTinyRotHexLook(use_pos_embed=True, directions=6, global_directions=12, angular_bins_per_radius=3,
                                   look_compact_variable_rings=True, tokenizer_null_initial_score=0.0)
        look = model.look_bank
        assert isinstance(look, SquarePatchDenseGridLook)
        with torch.no_grad():
            look.look_grid.copy_(torch.randn(look.look_grid.shape, generator=torch.Generator().manual_seed(3)))
            fields = look.transformed_look_grids()
        geometry = slot_geometry_of(look)
        assert geometry.slots.n_slots == 68 and geometry.planes == 12
        heads, n = fields.shape[0], geometry.patches
        flat = fields.reshape(heads, 12, n * n).double()
        values = flat[:, :, torch.from_numpy(geometry.representative)]
        table = torch.from_numpy(geometry.slots.table.astype(np.int64)).reshape(-1)
        none = table == 255
        rebuilt = values[:, :, table.masked_fill(none, 0)].masked_fill(none, 0.0)
        err = (rebuilt - flat).abs().max().item()
        assert err <= geometry.weight_error * look.look_grid.abs().max().item() + 1e-7
        assert geometry.weight_error <= 1e-5
    finally:
        sys.path.remove(str(REF))
        for key in [k for k in sys.modules if k.split(".")[0] in ("layers", "model", "utils")]:
            del sys.modules[key]
        sys.modules.update(saved)
