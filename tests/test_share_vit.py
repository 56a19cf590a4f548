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


def test_fused_gather_tables_reproduce_reflect_gather(model):
    """pixel_index / pixel_weight (read by the fused gather kernel) give exactly
    the reflect-padded, cover-weighted patches of both supports."""
    images = torch.randn(2, 3, 224, 224, generator=torch.Generator().manual_seed(5))
    ref = torch.cat([model._patches(images, 0), model._patches(images, 1)], dim=-1)
    got = images.flatten(1)[:, model.pixel_index.long()] * model.pixel_weight
    assert model.pixel_index.shape == (195, 3 * (448 + 112))
    assert int(model.pixel_index.min()) >= 0 and int(model.pixel_index.max()) < 3 * 224 * 224
    torch.testing.assert_close(got, ref, rtol=0, atol=0)


def test_fused_embed_weight_matrix_layout(model):
    """One GEMM against the fused matrix gives the tokenizer scores summed over
    both supports and the Look-bank responses of each support."""
    images = torch.randn(2, 3, 224, 224, generator=torch.Generator().manual_seed(6))
    p0, p1 = model._patches(images, 0).reshape(-1, 1344), model._patches(images, 1).reshape(-1, 336)
    w, fields = model._fused_embed_weights(torch.device("cpu"), torch.float32)
    mats = model._rendered(torch.device("cpu"), torch.float32)
    resp = torch.cat([p0, p1], dim=1) @ w.t()
    r0, r1 = p0 @ mats[0].t(), p1 @ mats[1].t()
    torch.testing.assert_close(resp[:, :576], r0[:, :576] + r1[:, :576], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(resp[:, 576:792], r0[:, 576:], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(resp[:, 792:], r1[:, 576:], rtol=1e-4, atol=1e-4)
    assert fields.shape == (36, 12, 68)


def test_gather_plan_reproduces_pixel_index(model):
    """Each group's sorted distinct 16-byte units, addressed by local_index,
    give back pixel_index; the model's groups fit the kernel's shared memory."""
    from intp_preliminary_b200.share_vit_ops import gather_plan
    for group in (1, 4, 13, 26):
        plan = gather_plan(model.pixel_index, group)
        index = model.pixel_index.long()
        begin = plan.stage_begin.tolist()
        assert len(begin) == -(-index.shape[0] // group) + 1 and begin[0] == 0
        for g in range(len(begin) - 1):
            units = plan.stage_offset[begin[g]:begin[g + 1]].long()
            assert torch.all(units[1:] > units[:-1])
            rows = slice(g * group, (g + 1) * group)
            local = plan.local_index[rows].long()
            assert torch.equal(4 * units[local // 4] + local % 4, index[rows])
        assert plan.max_stage == max(b - a for a, b in zip(begin[:-1], begin[1:]))
        assert plan.max_offset == int(index.max())
    assert model.gather_stage_begin.numel() - 1 == -(-model.num_patches // model._gather_plan_sizes[0])
    assert model._gather_plan_sizes[1] * 16 * 8 <= 228 * 1024  # 8 CTAs per SM


def test_gather_plan_rejects_bad_tables():
    from intp_preliminary_b200.share_vit_ops import gather_plan
    with pytest.raises(ValueError):
        gather_plan(torch.full((2, 8), -1, dtype=torch.int32))
    with pytest.raises(ValueError):
        gather_plan(torch.zeros(2, 6, dtype=torch.int32))
    with pytest.raises(ValueError):
        gather_plan(torch.zeros(2, 8, dtype=torch.int32), group_patches=0)
    with pytest.raises(ValueError):
        gather_plan(torch.arange(40000 * 8, dtype=torch.int32).reshape(40000, 8), group_patches=5000)  # 10000 units


def test_fused_op_wrappers_reject_cpu_tensors():
    from intp_preliminary_b200 import share_vit_ops as ops
    with pytest.raises(ValueError):
        ops.gather_patches(torch.zeros(1, 3, 8, 8), torch.zeros(2, 8, dtype=torch.int32), torch.zeros(8))
    with pytest.raises(ValueError):
        ops.add_layernorm(torch.zeros(4, 192), None, torch.ones(192), torch.zeros(192), 1e-6)
