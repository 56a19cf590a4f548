"""GPU parity of the backward passes (Look attention and negative L1) against the
reference's gradients (fixtures made by tests/golden/make_golden.py from the
reference's modules) and the float64 oracle.  Every call goes through
libintp_b200.so.

Tolerances follow the reference's own gradient tests
(tests/test_triton_structured_look_attention.py:61-141: fp32 3e-5, fp16 4e-3;
tests/test_triton_negative_l1.py:22-35: 2e-5)."""

import math

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import (LookSlots, check_device_status, hexgrid, look_attention_backward,
                                   look_attention_forward, negative_l1_distance, structured_look_attention)
from oracle.look_attention import reference_structured_look_attention
from tests.golden_data import load, tensor

pytestmark = pytest.mark.gpu
LOOK = load("look_attention_reference.npz")
NL1 = load("negative_l1_reference.npz")


def _case(prefix):
    return {k[len(prefix) + 1:]: v for k, v in LOOK.items() if k.startswith(prefix + "_")}


@pytest.fixture(autouse=True)
def _device_status(cuda_device):
    yield
    check_device_status(cuda_device)


@pytest.mark.parametrize("poses", [8, 18])
@pytest.mark.parametrize("dense", [False, True])
def test_all_gradients_match_reference_fp32(cuda_device, poses, dense):
    g = _case(f"p{poses}")
    leaves = [tensor(g[n]).to(cuda_device).requires_grad_(True) for n in ("q", "k", "v", "pose", "fields")]
    dense_t = tensor(g["dense"]).to(cuda_device).requires_grad_(True) if dense else None
    out = structured_look_attention(*leaves, scale=float(g["scale"]), dense_bias=dense_t)
    out.backward(tensor(g["grad_out"]).to(cuda_device))
    tag = "grad_dense" if dense else "grad"
    for name, leaf in zip(("q", "k", "v", "pose", "fields"), leaves):
        torch.testing.assert_close(leaf.grad.cpu(), tensor(g[f"{tag}_{name}"]), atol=3e-5, rtol=3e-5)
    if dense:
        torch.testing.assert_close(dense_t.grad.cpu(), tensor(g["grad_dense_dense"]), atol=3e-5, rtol=3e-5)


@pytest.mark.parametrize("poses", [8, 18])
def test_all_gradients_half_precision(cuda_device, poses):
    g = _case(f"p{poses}")
    inputs = [tensor(g[n]).half() for n in ("q", "k", "v", "pose", "fields")]
    leaves = [t.to(cuda_device).requires_grad_(True) for t in inputs]
    out = structured_look_attention(*leaves, scale=float(g["scale"]))
    grad_out = tensor(g["grad_out"]).half()
    out.backward(grad_out.to(cuda_device))
    # The reference's test accepts 4e-3 between its kernel and its oracle run in
    # half precision; that half oracle is itself up to ~3e-3 from the exact
    # gradients of the same (half) inputs.  Here: against the exact gradients
    # (float64), with both allowances, and never more than twice as far from them
    # as the half oracle is.
    exact = [t.double().requires_grad_(True) for t in inputs]
    ref = reference_structured_look_attention(*exact, scale=float(g["scale"]))
    ref.backward(grad_out.double())
    half_oracle = [t.clone().requires_grad_(True) for t in inputs]
    reference_structured_look_attention(*half_oracle, scale=float(g["scale"])).backward(grad_out)
    for leaf, ex, ho in zip(leaves, exact, half_oracle):
        assert leaf.grad.dtype == torch.float16
        ours = leaf.grad.cpu().double()
        torch.testing.assert_close(ours, ex.grad, atol=7e-3, rtol=4e-3)
        assert (ours - ex.grad).abs().max() <= 2 * (ho.grad.double() - ex.grad).abs().max() + 1e-3


def test_slot_gradients_match_reference_config1(cuda_device):
    """SLOTS mode (one-hot fields as a slot table): d(per-slot pose) is the
    reference's d(pose) through the one-hot fields."""
    g = _case("cfg1")
    q, k, v = (tensor(g[n]).to(cuda_device).requires_grad_(True) for n in ("q", "k", "v"))
    pose = tensor(g["pose"]).to(cuda_device).requires_grad_(True)
    slots = LookSlots(g["slots"], int(g["n_slots"]))
    out = structured_look_attention(q, k, v, pose, slots, scale=float(g["scale"]))
    out.backward(tensor(g["grad_out"]).to(cuda_device))
    for name, leaf in (("q", q), ("k", k), ("v", v), ("pose", pose)):
        ref = tensor(g[f"grad_{name}"])
        torch.testing.assert_close(leaf.grad.cpu(), ref, atol=1e-4, rtol=1e-4)


def test_bf16_slot_backward_after_tensor_core_forward(cuda_device):
    """bf16 forward on the tensor-core kernel (LSE from it), backward on CUDA cores,
    against float64 autograd through the oracle."""
    rows = cols = 12
    n_dir, n_rad = 8, 4
    slots = LookSlots(hexgrid.synthetic_look_slots(rows, cols, n_dir, n_rad), n_dir * n_rad)
    n = rows * cols + 1
    gen = torch.Generator().manual_seed(21)
    q, k, v = ((torch.randn(2, 3, n, 64, generator=gen) / 8).to(torch.bfloat16) for _ in range(3))
    pose = torch.rand(2, n - 1, 3, n_dir * n_rad, generator=gen) * 2 - 1
    grad_out = torch.randn(2, 3, n, 64, generator=gen).to(torch.bfloat16)
    leaves = [t.to(cuda_device).requires_grad_(True) for t in (q, k, v, pose)]
    out = structured_look_attention(*leaves[:4], slots, scale=0.125)
    out.backward(grad_out.to(cuda_device))
    onehot = torch.zeros(n_dir * n_rad, n - 1, n - 1, dtype=torch.float64)
    table = torch.from_numpy(slots.table.astype(np.int64))
    for s in range(n_dir * n_rad):
        onehot[s] = (table == s).double()
    fields = onehot.unsqueeze(0).expand(3, -1, -1, -1)
    ref_leaves = [t.double().requires_grad_(True) for t in (q, k, v, pose)]
    ref = reference_structured_look_attention(*ref_leaves, fields, scale=0.125)
    ref.backward(grad_out.double())
    for leaf, ref_leaf in zip(leaves, ref_leaves):
        err = (leaf.grad.cpu().double() - ref_leaf.grad).abs().max().item()
        assert err <= 2e-2 * max(ref_leaf.grad.abs().max().item(), 1e-3), err


def test_backward_entry_point_without_autograd(cuda_device):
    """look_attention_backward called directly: only the requested gradients."""
    g = _case("p8")
    q, k, v, pose, fields = (tensor(g[n]).to(cuda_device) for n in ("q", "k", "v", "pose", "fields"))
    out, lse = look_attention_forward(q, k, v, pose, fields, scale=float(g["scale"]), want_lse=True)
    grads = look_attention_backward(q, k, v, out, lse, tensor(g["grad_out"]).to(cuda_device), pose, fields,
                                    scale=float(g["scale"]), needs=(True, False, False, True, False, False))
    assert grads[1] is None and grads[2] is None and grads[4] is None and grads[5] is None
    torch.testing.assert_close(grads[0].cpu(), tensor(g["grad_q"]), atol=3e-5, rtol=3e-5)
    torch.testing.assert_close(grads[3].cpu(), tensor(g["grad_pose"]), atol=3e-5, rtol=3e-5)


@pytest.mark.parametrize("name", ["t7x11", "t37x67"])
def test_negative_l1_gradients_match_reference(cuda_device, name):
    x = torch.from_numpy(NL1[f"{name}_x"]).to(cuda_device).requires_grad_(True)
    w = torch.from_numpy(NL1[f"{name}_w"]).to(cuda_device).requires_grad_(True)
    out = negative_l1_distance(x, w)
    out.backward(torch.from_numpy(NL1[f"{name}_grad_out"]).to(cuda_device))
    torch.testing.assert_close(x.grad.cpu(), torch.from_numpy(NL1[f"{name}_grad_x"]), atol=2e-5, rtol=2e-5)
    torch.testing.assert_close(w.grad.cpu(), torch.from_numpy(NL1[f"{name}_grad_w"]), atol=2e-5, rtol=2e-5)


def test_negative_l1_gradient_sign_of_zero(cuda_device):
    """sign(0) = 0: identical rows contribute nothing (layers/triton_negative_l1.py:97-101)."""
    x = torch.tensor([[1.0, 2.0, 3.0]], device=cuda_device, requires_grad=True)
    w = torch.tensor([[1.0, 0.0, 5.0]], device=cuda_device, requires_grad=True)
    negative_l1_distance(x, w).backward(torch.ones(1, 1, device=cuda_device))
    assert x.grad.tolist() == [[0.0, -1.0, 1.0]]
    assert w.grad.tolist() == [[0.0, 1.0, -1.0]]


def test_negative_l1_gradients_at_tokenizer_scale(cuda_device):
    gen = torch.Generator().manual_seed(8)
    x = torch.randn(300, 336, generator=gen)
    w = torch.randn(96, 336, generator=gen) * 0.5
    go = torch.randn(300, 96, generator=gen)
    xd, wd = x.to(cuda_device).requires_grad_(True), w.to(cuda_device).requires_grad_(True)
    negative_l1_distance(xd, wd).backward(go.to(cuda_device))
    xr, wr = x.double().requires_grad_(True), w.double().requires_grad_(True)
    (-torch.cdist(xr, wr, p=1)).backward(go.double())
    torch.testing.assert_close(xd.grad.cpu().double(), xr.grad, atol=1e-3, rtol=1e-5)
    torch.testing.assert_close(wd.grad.cpu().double(), wr.grad, atol=1e-3, rtol=1e-5)


@pytest.mark.parametrize("head_dim", [20, 40, 96, 128])
def test_gradients_across_head_dims(cuda_device, head_dim):
    """The backward kernels are built per head-dim width (up to 32, 64 and 128
    lanes of accumulators) with the head dimension padded to a multiple of 4 in
    shared memory: every width and a padded one against float64 autograd through
    the oracle (general FIELDS form, fp32, the reference's 3e-5)."""
    g = torch.Generator().manual_seed(head_dim)
    b, h, patches, poses = 2, 2, 23, 5
    q, k, v = (torch.randn(b, h, patches + 1, head_dim, generator=g) / 4 for _ in range(3))
    pose = torch.randn(b, patches, h, poses, generator=g)
    fields = torch.randn(h, poses, patches, patches, generator=g) / 4
    grad = torch.randn(b, h, patches + 1, head_dim, generator=g)
    leaves = [t.to(cuda_device).requires_grad_(True) for t in (q, k, v, pose, fields)]
    out = structured_look_attention(*leaves, scale=1 / math.sqrt(head_dim))
    out.backward(grad.to(cuda_device))
    ref_leaves = [t.double().requires_grad_(True) for t in (q, k, v, pose, fields)]
    ref = reference_structured_look_attention(*ref_leaves, scale=1 / math.sqrt(head_dim))
    ref.backward(grad.double())
    torch.testing.assert_close(out.detach().cpu().double(), ref.detach(), atol=3e-5, rtol=3e-5)
    for leaf, ref_leaf in zip(leaves, ref_leaves):
        torch.testing.assert_close(leaf.grad.cpu().double(), ref_leaf.grad, atol=3e-5, rtol=3e-5)
