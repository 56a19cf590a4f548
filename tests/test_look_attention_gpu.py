"""GPU parity of the structured Look attention kernels against the oracle and
the reference's golden outputs.  Every call goes through libintp_b200.so.

Tolerances: the reference's own (fp32 2e-5, fp16 2e-3, tests/test_triton_structured_look_attention.py:60-141)
where its inputs are replayed; fp32 1e-4 max-abs and bf16 2e-2 max-abs for
the synthetic Look configurations, with tighter internal bars where they hold.
"""

import math

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import LookSlots, check_device_status, hexgrid, look_attention_forward
from intp_preliminary_b200 import structured_look_attention
from oracle.look_attention import look_attention_np, slot_look_attention_np
from tests.golden_data import load, tensor

pytestmark = pytest.mark.gpu
LOOK = load("look_attention_reference.npz")


def _case(prefix):
    return {k[len(prefix) + 1:]: v for k, v in LOOK.items() if k.startswith(prefix + "_")}


@pytest.fixture(autouse=True)
def _device_status(cuda_device):
    yield
    check_device_status(cuda_device)


@pytest.mark.parametrize("poses", [8, 18])
@pytest.mark.parametrize("dense", [False, True])
def test_reference_inputs_fp32(cuda_device, poses, dense):
    g = _case(f"p{poses}")
    q, k, v, pose, fields = (tensor(g[n]).to(cuda_device) for n in ("q", "k", "v", "pose", "fields"))
    dense_t = tensor(g["dense"]).to(cuda_device) if dense else None
    out = structured_look_attention(q, k, v, pose, fields, scale=float(g["scale"]), dense_bias=dense_t)
    expected = torch.from_numpy(g["out_dense"] if dense else g["out"])
    torch.testing.assert_close(out.cpu(), expected, atol=2e-5, rtol=2e-5)


@pytest.mark.parametrize("poses", [8, 18])
def test_reference_inputs_fp16(cuda_device, poses):
    g = _case(f"p{poses}")
    q, k, v, pose, fields = (tensor(g[n]).half().to(cuda_device) for n in ("q", "k", "v", "pose", "fields"))
    out = structured_look_attention(q, k, v, pose, fields, scale=float(g["scale"]))
    assert out.dtype == torch.float16
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(g["out_half"]), atol=2e-3, rtol=2e-3)


def test_config1_fp32_slots_and_fields(cuda_device):
    """14x14 hex lattice, 12 directions x 4 rings, fp32 (the B8 H3 N197 Look layer's lattice, B=1)."""
    g = _case("cfg1")
    q, k, v, pose = (tensor(g[n]).to(cuda_device) for n in ("q", "k", "v", "pose"))
    slots = LookSlots(g["slots"], int(g["n_slots"]))
    scale = float(g["scale"])
    expected = torch.from_numpy(g["out"])
    out_slots = structured_look_attention(q, k, v, pose, slots, scale=scale)
    torch.testing.assert_close(out_slots.cpu(), expected, atol=2e-5, rtol=2e-5)
    fields = slots.dense_fields(q.shape[1], device=cuda_device)
    out_fields = structured_look_attention(q, k, v, pose, fields, scale=scale)
    torch.testing.assert_close(out_fields.cpu(), expected, atol=2e-5, rtol=2e-5)
    assert (out_slots - out_fields).abs().max().item() <= 1e-4


def test_config4_bf16_golden(cuda_device):
    """32x32 hex lattice (N=1025), 8 directions x 4 rings, bf16 on tensor cores."""
    g = _case("cfg4")
    q, k, v = (tensor(g[n]).to(cuda_device) for n in ("q", "k", "v"))
    pose = tensor(g["pose"]).to(cuda_device)
    slots = LookSlots(g["slots"], int(g["n_slots"]))
    out, _ = look_attention_forward(q, k, v, pose, slots, scale=float(g["scale"]), kernel="tcgen05")
    golden = torch.from_numpy(g["out"])
    assert (out.float().cpu() - golden).abs().max().item() <= 2e-2
    exact = slot_look_attention_np(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                                   g["pose"], g["slots"], scale=float(g["scale"]))
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 1e-2


def _random_slot_inputs(batch, heads, rows, cols, n_dir, n_rad, dtype, device, seed=0):
    g = torch.Generator().manual_seed(seed)
    patches = rows * cols
    q, k, v = ((torch.randn(batch, heads, patches + 1, 64, generator=g) / 8).to(dtype) for _ in range(3))
    pose = torch.rand(batch, patches, heads, n_dir * n_rad, generator=g) * 2 - 1
    slots = hexgrid.synthetic_look_slots(rows, cols, n_dir, n_rad)
    return q.to(device), k.to(device), v.to(device), pose.to(device), slots


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols", [(1, 1), (1, 7), (8, 8), (14, 14), (9, 15), (16, 16), (8, 33)])
def test_tcgen05_slots_vs_oracle(cuda_device, dtype, rows, cols):
    q, k, v, pose, slots = _random_slot_inputs(2, 3, rows, cols, 12, 4, dtype, cuda_device, seed=rows * 100 + cols)
    look = LookSlots(slots, 48)
    out, lse = look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="tcgen05", want_lse=True)
    exact, exact_lse = slot_look_attention_np(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                              v.float().cpu().numpy(), pose.cpu().numpy(), slots,
                                              scale=0.125, return_lse=True)
    err = np.abs(out.float().cpu().numpy() - exact).max()
    assert err <= (8e-3 if dtype == torch.bfloat16 else 2e-3), err
    # The tensor-core path sums the 16-bit probabilities it multiplies into V
    # (row sum accumulated by the PV MMA), so the LSE carries their rounding.
    assert np.abs(lse.cpu().numpy() - exact_lse).max() <= (4e-3 if dtype == torch.bfloat16 else 1e-3)
    simt, _ = look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="simt")
    assert (out.float() - simt.float()).abs().max().item() <= 1e-2


@pytest.mark.parametrize("seq", [2, 3, 64, 65, 127, 128, 129, 200, 257])
def test_tcgen05_no_bias_odd_lengths(cuda_device, seq):
    g = torch.Generator().manual_seed(seq)
    q, k, v = ((torch.randn(3, 2, seq, 64, generator=g)).to(torch.bfloat16).to(cuda_device) for _ in range(3))
    pose = torch.zeros(3, seq - 1, 2, 1, device=cuda_device)
    fields = torch.zeros(2, 1, seq - 1, seq - 1, device=cuda_device)
    out_tc, _ = look_attention_forward(q, k, v, pose, LookSlots(np.full((seq - 1, seq - 1), 255, np.uint8), 1),
                                       scale=0.125, kernel="tcgen05")
    exact = look_attention_np(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                              pose.cpu().numpy(), fields.cpu().numpy(), scale=0.125)
    assert np.abs(out_tc.float().cpu().numpy() - exact).max() <= 2e-2


def test_strided_qkv_view(cuda_device):
    """q/k/v as the permuted view of one qkv projection (layers/mini_vit.py:69-71)."""
    batch, heads, rows, cols = 4, 3, 14, 14
    patches = rows * cols
    g = torch.Generator().manual_seed(5)
    qkv = (torch.randn(batch, patches + 1, 3, heads, 64, generator=g) / 8).to(torch.bfloat16).to(cuda_device)
    q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)
    assert not q.is_contiguous()
    pose = (torch.rand(batch, patches, heads, 48, generator=g) * 2 - 1).to(cuda_device)
    look = LookSlots(hexgrid.synthetic_look_slots(rows, cols, 12, 4), 48)
    out, _ = look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="tcgen05")
    ref, _ = look_attention_forward(q.contiguous(), k.contiguous(), v.contiguous(), pose, look, scale=0.125,
                                    kernel="tcgen05")
    torch.testing.assert_close(out, ref, atol=0, rtol=0)
    # pose as a strided per-layer slice of a wider pose tensor
    wide = (torch.rand(batch, patches, 3 * heads, 48, generator=g) * 2 - 1).to(cuda_device)
    layer_pose = wide[:, :, heads:2 * heads]
    out2, _ = look_attention_forward(q, k, v, layer_pose, look, scale=0.125, kernel="tcgen05")
    ref2, _ = look_attention_forward(q, k, v, layer_pose.contiguous(), look, scale=0.125, kernel="tcgen05")
    torch.testing.assert_close(out2, ref2, atol=0, rtol=0)


def test_config4_full_size_properties(cuda_device):
    """The long-sequence Look layer at full size (B64, H6, N1025, bf16): oracle on a sampled
    subset of (batch, head) pairs, finiteness and run-to-run determinism."""
    batch, heads, rows, cols = 64, 6, 32, 32
    q, k, v, pose, slots = _random_slot_inputs(batch, heads, rows, cols, 8, 4, torch.bfloat16, cuda_device, seed=7)
    look = LookSlots(slots, 32)
    out1, _ = look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="tcgen05")
    out2, _ = look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="tcgen05")
    assert torch.isfinite(out1.float()).all()
    assert torch.equal(out1, out2)
    for b, h in [(0, 0), (17, 3), (63, 5)]:
        exact = slot_look_attention_np(q[b:b + 1, h:h + 1].float().cpu().numpy(), k[b:b + 1, h:h + 1].float().cpu().numpy(),
                                       v[b:b + 1, h:h + 1].float().cpu().numpy(),
                                       pose[b:b + 1, :, h:h + 1].cpu().numpy(), slots, scale=0.125)
        assert np.abs(out1[b:b + 1, h:h + 1].float().cpu().numpy() - exact).max() <= 2e-2


def test_general_fields_bf16_simt_matches_oracle(cuda_device):
    g = torch.Generator().manual_seed(11)
    batch, heads, patches, poses = 2, 3, 40, 12
    q, k, v = ((torch.randn(batch, heads, patches + 1, 64, generator=g) / 8).to(torch.bfloat16) for _ in range(3))
    pose = torch.rand(batch, patches, heads, poses, generator=g)
    fields = torch.randn(heads, poses, patches, patches, generator=g) * 0.1
    dense = torch.randn(batch, heads, patches, patches, generator=g) * 0.1
    out = structured_look_attention(*(t.to(cuda_device) for t in (q, k, v, pose, fields)), scale=0.125,
                                    dense_bias=dense.to(cuda_device))
    exact = look_attention_np(q.float().numpy(), k.float().numpy(), v.float().numpy(), pose.numpy(), fields.numpy(),
                              scale=0.125, dense_bias=dense.numpy())
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 1e-2


def test_tcgen05_refuses_what_it_cannot_take(cuda_device):
    q = torch.randn(1, 1, 9, 32, device=cuda_device, dtype=torch.bfloat16)
    pose = torch.zeros(1, 8, 1, 1, device=cuda_device)
    look = LookSlots(np.full((8, 8), 255, np.uint8), 1)
    with pytest.raises(RuntimeError):
        look_attention_forward(q, q, q, pose, look, scale=0.1, kernel="tcgen05")
    out, _ = look_attention_forward(q, q, q, pose, look, scale=0.1, kernel="auto")
    assert out.shape == q.shape


def test_shape_errors_match_reference_messages(cuda_device):
    q = torch.randn(1, 1, 5, 16, device=cuda_device)
    with pytest.raises(ValueError, match="patch_count"):
        structured_look_attention(q, q, q, torch.randn(1, 3, 1, 2, device=cuda_device),
                                  torch.randn(1, 2, 3, 3, device=cuda_device), scale=1.0)
    with pytest.raises(ValueError, match="fields shape"):
        structured_look_attention(q, q, q, torch.randn(1, 4, 1, 2, device=cuda_device),
                                  torch.randn(1, 3, 4, 4, device=cuda_device), scale=1.0)
    with pytest.raises(ValueError, match="head_dim"):
        big = torch.randn(1, 1, 5, 160, device=cuda_device)
        structured_look_attention(big, big, big, torch.randn(1, 4, 1, 2, device=cuda_device),
                                  torch.randn(1, 2, 4, 4, device=cuda_device), scale=1.0)


def test_empty_batch(cuda_device):
    q = torch.randn(0, 2, 9, 64, device=cuda_device, dtype=torch.bfloat16)
    out = structured_look_attention(q, q, q, torch.zeros(0, 8, 2, 4, device=cuda_device),
                                    torch.zeros(2, 4, 8, 8, device=cuda_device), scale=0.125)
    assert out.shape == q.shape


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("patches,poses,dense", [(40, 12, True), (40, 18, False), (129, 1, True), (195, 18, True),
                                                 (255, 6, False), (5, 3, True)])
def test_tcgen05_general_fields_and_dense_vs_oracle(cuda_device, dtype, patches, poses, dense):
    """The reference's general form - dense (H, P, Np, Np) fields and a dense
    (B, H, Np, Np) bias, as the dual-Look model (P = 12 + 6) and the grid-first
    variants pass them - on the tensor-core kernel (N <= 256)."""
    g = torch.Generator().manual_seed(patches * 7 + poses)
    batch, heads = 2, 3
    q, k, v = ((torch.randn(batch, heads, patches + 1, 64, generator=g) / 8).to(dtype) for _ in range(3))
    pose = torch.rand(batch, patches, heads, poses, generator=g)
    fields = torch.randn(heads, poses, patches, patches, generator=g) * 0.3
    dense_t = torch.randn(batch, heads, patches, patches, generator=g) * 0.3 if dense else None
    out, lse = look_attention_forward(*(t.to(cuda_device) for t in (q, k, v, pose, fields)), scale=0.125,
                                      dense_bias=dense_t.to(cuda_device) if dense else None, kernel="tcgen05",
                                      want_lse=True)
    exact, exact_lse = look_attention_np(q.float().numpy(), k.float().numpy(), v.float().numpy(), pose.numpy(),
                                         fields.numpy(), scale=0.125,
                                         dense_bias=dense_t.numpy() if dense else None, return_lse=True)
    err = np.abs(out.float().cpu().numpy() - exact).max()
    assert err <= (8e-3 if dtype == torch.bfloat16 else 2e-3), err
    assert np.abs(lse.cpu().numpy() - exact_lse).max() <= 1e-3
