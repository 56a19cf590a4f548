"""The oracle against golden vectors produced by the reference itself (CPU)."""

import numpy as np
import pytest
import torch

from oracle import hex_lattice
from oracle.look_attention import (
    look_attention_np,
    onehot_fields,
    reference_structured_look_attention,
    slot_look_attention_np,
)
from oracle.negative_l1 import negative_l1_np, negative_l1_torch
from tests.golden_data import load, tensor

LOOK = load("look_attention_reference.npz")
NL1 = load("negative_l1_reference.npz")
HEX = load("hex_bins_reference.npz")


@pytest.mark.parametrize("poses", [8, 18])
@pytest.mark.parametrize("dense", [False, True])
def test_torch_oracle_matches_reference_test_inputs(poses, dense):
    g = {k[len(f"p{poses}_"):]: v for k, v in LOOK.items() if k.startswith(f"p{poses}_")}
    args = [tensor(g[n]) for n in ("q", "k", "v", "pose", "fields")]
    out = reference_structured_look_attention(
        *args, scale=float(g["scale"]), dense_bias=tensor(g["dense"]) if dense else None
    )
    expected = g["out_dense"] if dense else g["out"]
    np.testing.assert_allclose(out.numpy(), expected, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("poses", [8, 18])
def test_numpy_oracle_matches_reference(poses):
    g = {k[len(f"p{poses}_"):]: v for k, v in LOOK.items() if k.startswith(f"p{poses}_")}
    for dense in (None, g["dense"]):
        out = look_attention_np(g["q"], g["k"], g["v"], g["pose"], g["fields"], scale=float(g["scale"]),
                                dense_bias=dense)
        expected = g["out"] if dense is None else g["out_dense"]
        np.testing.assert_allclose(out, expected, rtol=2e-5, atol=2e-5)


def test_half_golden_is_close_to_fp32():
    g = {k[3:]: v for k, v in LOOK.items() if k.startswith("p8_")}
    np.testing.assert_allclose(g["out_half"], g["out"], atol=5e-3)


@pytest.mark.parametrize("cfg", ["cfg1", "cfg4"])
def test_slot_oracle_matches_reference_onehot(cfg):
    g = {k[len(cfg) + 1:]: v for k, v in LOOK.items() if k.startswith(cfg + "_")}
    q, k, v = (tensor(g[n]).float().numpy() for n in ("q", "k", "v"))
    out = slot_look_attention_np(q, k, v, g["pose"], g["slots"], scale=float(g["scale"]))
    tol = 1e-5 if cfg == "cfg1" else 1e-2  # cfg4 golden is the reference's bf16 output
    np.testing.assert_allclose(out, g["out"], atol=tol, rtol=tol)


def test_cfg1_slot_table_is_the_oracle_table():
    g = {k[5:]: v for k, v in LOOK.items() if k.startswith("cfg1_")}
    table = np.asarray(hex_lattice.slot_table(hex_lattice.lattice_points(14, 14), 12, 4), dtype=np.uint8)
    np.testing.assert_array_equal(table, g["slots"])
    # ring-1 neighbours only lie at multiples of 60 degrees, so the six odd
    # 30-degree directions never carry a ring-1 pair: 42 of 48 slots occur.
    unused = {d * 4 for d in range(1, 12, 2)}
    assert set(np.unique(table[table != 255]).tolist()) == set(range(48)) - unused


def test_onehot_fields_equal_slot_gather():
    g = {k[5:]: v for k, v in LOOK.items() if k.startswith("cfg1_")}
    fields = onehot_fields(g["slots"], int(g["n_slots"]), heads=3)
    a = look_attention_np(g["q"], g["k"], g["v"], g["pose"], fields, scale=float(g["scale"]))
    b = slot_look_attention_np(g["q"], g["k"], g["v"], g["pose"], g["slots"], scale=float(g["scale"]))
    np.testing.assert_allclose(a, b, atol=1e-12)


@pytest.mark.parametrize("name", ["t7x11", "t37x67", "b432", "b1728"])
def test_negative_l1_oracle_matches_reference(name):
    x, w, expected = NL1[f"{name}_x"], NL1[f"{name}_w"], NL1[f"{name}_out"]
    np.testing.assert_allclose(negative_l1_np(x, w), expected, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(negative_l1_torch(torch.from_numpy(x), torch.from_numpy(w)).numpy(), expected,
                               rtol=1e-6, atol=1e-5)


@pytest.mark.parametrize("prefix", ["lattice14", "real"])
def test_hex_oracle_matches_reference_bins(prefix):
    """Rings match exactly.  Directions match exactly except for pairs lying on a
    sector edge (angle an odd multiple of 30 degrees), where the reference's
    float32 atan2 rounds either way; there either neighbouring sector is accepted."""
    points = [tuple(p) for p in HEX[f"{prefix}_xy"].astype(np.float64)]
    rings = np.array([[hex_lattice.ring(a, b) for b in points] for a in points])
    dirs = np.array([[hex_lattice.six_sector(a, b) for b in points] for a in points])
    np.testing.assert_array_equal(rings, HEX[f"{prefix}_rings"])
    ref = HEX[f"{prefix}_dirs"].astype(np.int64)
    xy = np.asarray(points)
    delta = xy[None, :, :] - xy[:, None, :]
    sector_pos = (np.arctan2(delta[..., 1], delta[..., 0]) + np.pi / 6) / (np.pi / 3)
    on_edge = (np.abs(sector_pos - np.round(sector_pos)) < 1e-5) & (rings > 0)
    np.testing.assert_array_equal(dirs[~on_edge], ref[~on_edge])
    edge_gap = np.minimum(np.abs(dirs - ref), 6 - np.abs(dirs - ref))[on_edge]
    assert edge_gap.max(initial=0) <= 1
