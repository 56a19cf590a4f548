"""SHARE-ViT half6d3r model glue (CPU): geometry, state_dict layout, and the full
forward against the reference's logits with the attention kernel replaced by
the oracle (the kernel itself is checked by the GPU tests)."""

import numpy as np
import pytest
import torch

import intp_preliminary_b200.share_vit as sv
from oracle.look_attention import slot_look_attention_np
from tests.golden_data import load

GOLD = load("share_vit_reference.npz")


@pytest.fixture(scope="module")
def model():
    return sv.ShareViTHalf6d3r(precision="fp32").init_weights(seed=int(GOLD["weight_seed"]),
                                                              look_grid_std=float(GOLD["look_grid_std"]))


def test_geometry(model):
    assert model.num_patches == 195
    assert [s.samples for s in model.supports] == [448, 112]
    assert model.look_slots.n_slots == 68
    assert model.look_basis.shape == (12, 48, 68)
    valid = (model.look_slots.table != 255).sum(axis=1)
    assert valid.max() <= 61 and valid.min() >= 10


def test_state_dict_names_match_reference_layout(model):
    sd = model.state_dict()
    assert len(sd) == 158
    assert sd["patch_embed.prototype"].shape == (96, 3, 234)
    assert sd["look_bank.look_grid"].shape == (36, 4, 12)
    assert sd["look_bank.patch_coordinates_xy"].shape == (195, 2)
    assert sd["pos_embed"].shape == (1, 196, 192)
    clone = sv.ShareViTHalf6d3r(precision="fp32")
    clone.load_state_dict(sd, strict=True)


def _oracle_attention(q, k, v, pose, fields, *, scale, out=None, **_):
    out = slot_look_attention_np(q.double().numpy(), k.double().numpy(), v.double().numpy(), pose.double().numpy(),
                                 fields.table, scale=scale)
    return torch.from_numpy(out).to(q.dtype), None


def test_forward_glue_matches_reference_logits(model, monkeypatch):
    monkeypatch.setattr(sv, "look_attention_forward", _oracle_attention)
    images = torch.randn(2, 3, 224, 224, generator=torch.Generator().manual_seed(int(GOLD["image_seed"])))
    logits = model(images)
    np.testing.assert_allclose(logits.numpy(), GOLD["logits"], atol=1e-4, rtol=1e-4)


def test_seeded_init_is_deterministic():
    a = sv.ShareViTHalf6d3r(precision="fp32").init_weights(seed=3)
    b = sv.ShareViTHalf6d3r(precision="fp32").init_weights(seed=3)
    for (na, pa), (nb, pb) in zip(a.named_parameters(), b.named_parameters()):
        assert na == nb and torch.equal(pa, pb)


def test_cpu_port_matches_reference_logits(model):
    """The CPU baseline (dense fields + explicit oracle per layer) reproduces the
    reference's logits, so the timed CPU path computes the same thing."""
    from oracle.share_vit_cpu import reference_forward_cpu

    images = torch.randn(2, 3, 224, 224, generator=torch.Generator().manual_seed(int(GOLD["image_seed"])))
    np.testing.assert_allclose(reference_forward_cpu(model, images).numpy(), GOLD["logits"], atol=1e-4, rtol=1e-4)
