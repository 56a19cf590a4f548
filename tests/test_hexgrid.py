"""Product-side slot-table builder (host logic) against the oracle and the reference."""

import numpy as np
import pytest

from intp_preliminary_b200 import hexgrid
from oracle import hex_lattice
from tests.golden_data import load

HEX = load("hex_bins_reference.npz")


@pytest.mark.parametrize("rows,cols,n_dir,n_rad", [(14, 14, 12, 4), (5, 7, 8, 4), (6, 6, 12, 2), (3, 4, 6, 3)])
def test_slot_table_matches_oracle(rows, cols, n_dir, n_rad):
    product = hexgrid.synthetic_look_slots(rows, cols, n_dir, n_rad)
    oracle = np.asarray(hex_lattice.slot_table(hex_lattice.lattice_points(rows, cols), n_dir, n_rad), np.uint8)
    np.testing.assert_array_equal(product, oracle)


def test_cfg1_golden_slots():
    look = load("look_attention_reference.npz")
    np.testing.assert_array_equal(hexgrid.synthetic_look_slots(14, 14, 12, 4), look["cfg1_slots"])
    np.testing.assert_array_equal(hexgrid.synthetic_look_slots(32, 32, 8, 4), look["cfg4_slots"])


@pytest.mark.parametrize("prefix", ["lattice14", "real"])
def test_rings_match_reference(prefix):
    rings = hexgrid.hex_rings(HEX[f"{prefix}_xy"])
    np.testing.assert_array_equal(rings, HEX[f"{prefix}_rings"])


def test_lattice_is_offset_rows():
    xy = hexgrid.offset_row_lattice(2, 3)
    np.testing.assert_allclose(xy[:3, 0], [0, 1, 2])
    np.testing.assert_allclose(xy[3:, 0], [0.5, 1.5, 2.5])
    np.testing.assert_allclose(xy[3:, 1], np.sqrt(3) / 2)


def test_slot_table_properties():
    slots = hexgrid.synthetic_look_slots(32, 32, 8, 4)
    assert slots.shape == (1024, 1024)
    assert (np.diag(slots) == hexgrid.SLOT_NONE).all()
    # every query has at most 60 neighbours within ring 4 (6 + 12 + 18 + 24)
    assert ((slots != hexgrid.SLOT_NONE).sum(axis=1) <= 60).all()
    assert (slots[slots != hexgrid.SLOT_NONE] < 32).all()


def test_bad_arguments():
    with pytest.raises(ValueError):
        hexgrid.offset_row_lattice(0, 3)
    with pytest.raises(ValueError):
        hexgrid.direction_radius_slots(hexgrid.offset_row_lattice(2, 2), 100, 4)
