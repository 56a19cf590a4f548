"""GPU parity of the tensor-core Look attention on sequences longer than 256
tokens (the tiled kernel: online softmax over 64-key tiles, SLOTS Look bias or
none) against the float64 oracle.

The cases cover: query-tile counts that leave a partial last tile, last key
tiles of 1, 44 and 12 keys (the packed pair table masks the padding keys),
lengths that are multiples of 64 and 128, strided q/k/v views and a
token-major output view, and logits large enough that the running row max
moves (O rescaled in TMEM), both from one key tile to the next and within the
first tiles.  A share of the exponentials runs on the FMA pipe (a polynomial
with relative error <= 7.5e-5), so these cases also pin that path, masked keys
(-inf) included.  Tolerances: bf16 2e-2 max-abs on the outputs (the bf16 bar
for the synthetic Look configurations; met at 8e-3 here), f16 2e-3.
"""

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import LookSlots, check_device_status, hexgrid, look_attention_forward
from oracle.look_attention import look_attention_np, slot_look_attention_np

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device_status(cuda_device):
    yield
    check_device_status(cuda_device)


def _slot_inputs(batch, heads, rows, cols, n_dir, dtype, device, seed, qk_scale=1.0 / 8):
    g = torch.Generator().manual_seed(seed)
    patches = rows * cols
    q, k = ((torch.randn(batch, heads, patches + 1, 64, generator=g) * qk_scale).to(dtype) for _ in range(2))
    v = (torch.randn(batch, heads, patches + 1, 64, generator=g) / 8).to(dtype)
    pose = torch.rand(batch, patches, heads, n_dir * 4, generator=g) * 2 - 1
    slots = hexgrid.synthetic_look_slots(rows, cols, n_dir, 4)
    return q.to(device), k.to(device), v.to(device), pose.to(device), slots


def _oracle(q, k, v, pose, slots, scale=0.125):
    return slot_look_attention_np(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                                  pose.cpu().numpy(), slots, scale=scale, return_lse=True)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols", [(16, 16), (13, 23), (16, 32), (32, 32), (7, 157), (24, 24)])
def test_pair_slots_vs_oracle(cuda_device, dtype, rows, cols):
    """N = 257, 300, 513, 1025, 1100, 577 with an 8 x 4 Look field (32 slots)."""
    q, k, v, pose, slots = _slot_inputs(2, 3, rows, cols, 8, dtype, cuda_device, seed=rows * 1000 + cols)
    out, lse = look_attention_forward(q, k, v, pose, LookSlots(slots, 32), scale=0.125, kernel="tcgen05",
                                      want_lse=True)
    exact, exact_lse = _oracle(q, k, v, pose, slots)
    err = np.abs(out.float().cpu().numpy() - exact).max()
    assert err <= (8e-3 if dtype == torch.bfloat16 else 2e-3), err
    # the row sum is accumulated from the 16-bit probabilities the PV MMA multiplies
    assert np.abs(lse.cpu().numpy() - exact_lse).max() <= (4e-3 if dtype == torch.bfloat16 else 1e-3)


@pytest.mark.parametrize("seq", [258, 300, 384, 513, 1025, 1100])
def test_pair_no_bias(cuda_device, seq):
    g = torch.Generator().manual_seed(seq)
    q, k, v = ((torch.randn(2, 3, seq, 64, generator=g) / 4).to(torch.bfloat16).to(cuda_device) for _ in range(3))
    pose = torch.zeros(2, seq - 1, 3, 1, device=cuda_device)
    out, lse = look_attention_forward(q, k, v, pose, LookSlots(np.full((seq - 1, seq - 1), 255, np.uint8), 1),
                                      scale=0.125, kernel="tcgen05", want_lse=True)
    fields = np.zeros((3, 1, seq - 1, seq - 1), np.float32)
    exact = look_attention_np(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                              pose.cpu().numpy(), fields, scale=0.125)
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 8e-3


def test_pair_large_logits_rescale(cuda_device):
    """q, k ~ N(0, 1): logits spread over tens of units in the log2 domain, so
    the reference max moves inside and across key tiles."""
    q, k, v, pose, slots = _slot_inputs(2, 2, 32, 32, 8, torch.bfloat16, cuda_device, seed=3, qk_scale=1.0)
    pose = pose * 4
    out, lse = look_attention_forward(q, k, v, pose, LookSlots(slots, 32), scale=0.125, kernel="tcgen05",
                                      want_lse=True)
    exact, exact_lse = _oracle(q, k, v, pose, slots)
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 2e-2
    assert np.abs(lse.cpu().numpy() - exact_lse).max() <= 2e-2


def test_pair_max_grows_across_tiles(cuda_device):
    """Keys ordered so that each row's largest logits come in its last key
    tiles: the reference max moves after O has accumulated several tiles."""
    g = torch.Generator().manual_seed(4)
    seq = 1025
    q = (torch.randn(1, 2, seq, 64, generator=g)).to(torch.bfloat16)
    base = torch.randn(64, generator=g)
    # keys aligned with a shared direction, their strength growing with the key index
    strength = torch.linspace(0.0, 3.0, seq)[None, None, :, None]
    k = (strength * base + 0.3 * torch.randn(1, 2, seq, 64, generator=g)).to(torch.bfloat16)
    q = (q.float() * 0.3 + base).to(torch.bfloat16)
    v = (torch.randn(1, 2, seq, 64, generator=g) / 8).to(torch.bfloat16)
    q, k, v = (t.to(cuda_device) for t in (q, k, v))
    pose = torch.zeros(1, seq - 1, 2, 1, device=cuda_device)
    out, lse = look_attention_forward(q, k, v, pose, LookSlots(np.full((seq - 1, seq - 1), 255, np.uint8), 1),
                                      scale=0.125, kernel="tcgen05", want_lse=True)
    fields = np.zeros((2, 1, seq - 1, seq - 1), np.float32)
    exact, exact_lse = look_attention_np(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                                         pose.cpu().numpy(), fields, scale=0.125, return_lse=True)
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 2e-2
    assert np.abs(lse.cpu().numpy() - exact_lse).max() <= 2e-2


def test_pair_strided_views(cuda_device):
    """q/k/v as the permuted view of one (B, N, 3, H, D) projection and the
    output written into a token-major buffer, at N = 1025."""
    batch, heads, rows, cols = 2, 3, 32, 32
    patches = rows * cols
    g = torch.Generator().manual_seed(21)
    qkv = (torch.randn(batch, patches + 1, 3, heads, 64, generator=g) / 8).to(torch.bfloat16).to(cuda_device)
    q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)
    pose = (torch.rand(batch, patches, heads, 32, generator=g) * 2 - 1).to(cuda_device)
    look = LookSlots(hexgrid.synthetic_look_slots(rows, cols, 8, 4), 32)
    token_major = torch.empty(batch, patches + 1, heads, 64, dtype=torch.bfloat16, device=cuda_device)
    out_view = token_major.permute(0, 2, 1, 3)
    look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="tcgen05", out=out_view)
    ref, _ = look_attention_forward(q.contiguous(), k.contiguous(), v.contiguous(), pose, look, scale=0.125,
                                    kernel="tcgen05")
    torch.testing.assert_close(out_view, ref, atol=0, rtol=0)


def test_pair_matches_cuda_core_kernel_and_repeats(cuda_device):
    q, k, v, pose, slots = _slot_inputs(3, 2, 16, 32, 8, torch.bfloat16, cuda_device, seed=9)
    look = LookSlots(slots, 32)
    out1, _ = look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="tcgen05")
    out2, _ = look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="tcgen05")
    assert torch.equal(out1, out2)
    simt, _ = look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="simt")
    assert (out1.float() - simt.float()).abs().max().item() <= 1e-2
