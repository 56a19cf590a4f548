"""GPU parity of the SLOT_FIELDS Look form (``LookSlotFields``): the reference's
general fields call (layers/triton_structured_look_attention.py:25-54) with
fields that are per-slot values gathered by a pair table, as the reference
model's Look bank builds them (model/deit_tiny_rot_hex_look.py:397-451).
Checked against the float64 oracle on the expanded (H, P, Np, Np) fields.

Tolerances: fp32 1e-4 max-abs, bf16 2e-2 max-abs (tighter internal bars where
they hold), gradients as in test_backward_gpu.py."""

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import (LookSlotFields, LookSlots, check_device_status, hexgrid, look_attention_forward,
                                   structured_look_attention)
from oracle.look_attention import look_attention_np, reference_structured_look_attention, slot_fields_dense_np

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device_status(cuda_device):
    yield
    check_device_status(cuda_device)


def _inputs(batch, heads, rows, cols, n_dir, n_rad, poses, dtype, device, seed):
    g = torch.Generator().manual_seed(seed)
    patches = rows * cols
    q, k, v = ((torch.randn(batch, heads, patches + 1, 64, generator=g) / 8).to(dtype) for _ in range(3))
    pose = torch.softmax(torch.randn(batch, patches, heads, poses, generator=g), dim=-1)
    values = torch.randn(heads, poses, n_dir * n_rad, generator=g)
    slots = hexgrid.synthetic_look_slots(rows, cols, n_dir, n_rad)
    return [t.to(device) for t in (q, k, v, pose, values)] + [slots]


def _oracle(q, k, v, pose, values, slots, scale):
    fields = slot_fields_dense_np(values.cpu().numpy(), slots, dtype=np.float64)
    return look_attention_np(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                             pose.cpu().numpy(), fields, scale=scale, return_lse=True)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols,n_dir", [(1, 1, 6), (8, 8, 12), (14, 14, 17), (9, 15, 12), (8, 33, 6)])
def test_tcgen05_slot_fields_vs_oracle(cuda_device, dtype, rows, cols, n_dir):
    q, k, v, pose, values, slots = _inputs(2, 3, rows, cols, n_dir, 4, 12, dtype, cuda_device, rows * 31 + cols)
    look = LookSlotFields(LookSlots(slots, n_dir * 4), values)
    out, lse = look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="tcgen05", want_lse=True)
    exact, exact_lse = _oracle(q, k, v, pose, values, slots, 0.125)
    err = np.abs(out.float().cpu().numpy() - exact).max()
    assert err <= (8e-3 if dtype == torch.bfloat16 else 2e-3), err
    assert np.abs(lse.cpu().numpy() - exact_lse).max() <= (4e-3 if dtype == torch.bfloat16 else 1e-3)


@pytest.mark.parametrize("rows,cols", [(3, 5), (14, 14)])
def test_simt_slot_fields_fp32_vs_oracle(cuda_device, rows, cols):
    q, k, v, pose, values, slots = _inputs(2, 3, rows, cols, 12, 4, 12, torch.float32, cuda_device, 7 + rows)
    look = LookSlotFields(LookSlots(slots, 48), values)
    out, lse = look_attention_forward(q, k, v, pose, look, scale=0.125, want_lse=True)
    exact, exact_lse = _oracle(q, k, v, pose, values, slots, 0.125)
    assert np.abs(out.cpu().numpy() - exact).max() <= 1e-4
    assert np.abs(lse.cpu().numpy() - exact_lse).max() <= 1e-4


def test_slot_fields_equal_slots_with_materialised_values(cuda_device):
    """The two compact forms of the same fields give the same attention."""
    q, k, v, pose, values, slots = _inputs(4, 3, 14, 14, 17, 4, 12, torch.bfloat16, cuda_device, 5)
    table = LookSlots(slots, 68)
    per_slot = torch.einsum("bqhp,hps->bqhs", pose, values).contiguous()
    a, lse_a = look_attention_forward(q, k, v, pose, LookSlotFields(table, values), scale=0.125, want_lse=True)
    b, lse_b = look_attention_forward(q, k, v, per_slot, table, scale=0.125, want_lse=True)
    assert (a.float() - b.float()).abs().max().item() <= 4e-3
    assert (lse_a - lse_b).abs().max().item() <= 1e-3


def test_slot_fields_scalar_path_for_strided_values(cuda_device):
    """Slot values that are not 16-byte rows take the scalar table build."""
    q, k, v, pose, values, slots = _inputs(2, 3, 6, 7, 6, 4, 5, torch.bfloat16, cuda_device, 9)
    strided = values.transpose(0, 1).contiguous().transpose(0, 1)  # (H, P, S) with P outermost in memory
    assert strided.stride(0) != values.stride(0)
    out, _ = look_attention_forward(q, k, v, pose, LookSlotFields(LookSlots(slots, 24), strided), scale=0.125,
                                    kernel="tcgen05")
    exact, _ = _oracle(q, k, v, pose, values, slots, 0.125)
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 8e-3


def test_model_layout_pose_view(cuda_device):
    """Pose as the model passes it: a 3-head slice of a (B, Np, 36, 12) buffer,
    slot values a 3-head slice of (36, 12, S)."""
    q, k, v, _, _, slots = _inputs(3, 3, 14, 14, 17, 4, 12, torch.bfloat16, cuda_device, 13)
    g = torch.Generator().manual_seed(14)
    pose_all = torch.softmax(torch.randn(3, 196, 36, 12, generator=g), dim=-1).to(cuda_device)
    values_all = torch.randn(36, 12, 68, generator=g).to(cuda_device)
    pose, values = pose_all[:, :, 6:9], values_all[6:9]
    out, _ = look_attention_forward(q, k, v, pose, LookSlotFields(LookSlots(slots, 68), values), scale=0.125)
    exact, _ = _oracle(q, k, v, pose, values, slots, 0.125)
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 8e-3


def test_slot_fields_gradients_fp32(cuda_device):
    """Autograd through LookSlotFields against float64 autograd of the reference
    algorithm on the expanded fields."""
    q, k, v, pose, values, slots = _inputs(2, 2, 4, 5, 6, 2, 4, torch.float32, cuda_device, 21)
    table = LookSlots(slots, 12)
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v, pose, values)]
    out = structured_look_attention(*leaves[:4], LookSlotFields(table, leaves[4]), scale=0.125)
    g = torch.Generator().manual_seed(22)
    grad = torch.randn(out.shape, generator=g).to(cuda_device)
    out.backward(grad)
    ref_leaves = [t.detach().cpu().double().requires_grad_(True) for t in (q, k, v, pose, values)]
    none = torch.from_numpy(slots == 255)
    index = torch.from_numpy(np.where(slots == 255, 0, slots).astype(np.int64))
    fields = ref_leaves[4][:, :, index].masked_fill(none, 0.0)
    ref = reference_structured_look_attention(*ref_leaves[:4], fields, scale=0.125)
    ref.backward(grad.cpu().double())
    torch.testing.assert_close(out.detach().cpu().double(), ref.detach(), atol=1e-5, rtol=1e-5)
    for leaf, ref_leaf in zip(leaves, ref_leaves):
        torch.testing.assert_close(leaf.grad.cpu().double(), ref_leaf.grad, atol=1e-4, rtol=1e-4)
