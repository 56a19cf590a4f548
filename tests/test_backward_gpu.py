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
    """bf16 forward on the tensor-core kernel (LSE from it), backward (the tensor-core pass),
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


def _slot_case(rows, cols, n_dir, n_rad, batch, heads, dtype, seed):
    slots = LookSlots(hexgrid.synthetic_look_slots(rows, cols, n_dir, n_rad), n_dir * n_rad)
    n = rows * cols + 1
    gen = torch.Generator().manual_seed(seed)
    q, k, v = ((torch.randn(batch, heads, n, 64, generator=gen) / 8).to(dtype) for _ in range(3))
    pose = torch.rand(batch, n - 1, heads, n_dir * n_rad, generator=gen) * 2 - 1
    grad_out = torch.randn(batch, heads, n, 64, generator=gen).to(dtype)
    return slots, q, k, v, pose, grad_out


def _onehot_fields(slots, heads):
    n_slots = slots.n_slots
    table = torch.from_numpy(slots.table.astype(np.int64))
    onehot = torch.stack([(table == s).double() for s in range(n_slots)])
    return onehot.unsqueeze(0).expand(heads, -1, -1, -1)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("grid", [(14, 14, 12, 6), (20, 20, 8, 4), (3, 5, 4, 2)])
def test_tensor_core_backward_matches_oracle(cuda_device, dtype, grid):
    """The tensor-core backward (probability / score-gradient pass on tcgen05,
    then batched GEMMs) against float64 autograd through the oracle: the model's
    197 tokens with 72 slots, 401 tokens (4 query tiles, 7 key tiles, ragged
    ends) and a 16-token case.  Bar: 2 % of the largest gradient, the bf16 bar
    of the CUDA-core backward test above."""
    rows, cols, n_dir, n_rad = grid
    slots, q, k, v, pose, grad_out = _slot_case(rows, cols, n_dir, n_rad, 2, 3, dtype, seed=rows * 7 + n_dir)
    dev = [t.to(cuda_device) for t in (q, k, v, pose)]
    out, lse = look_attention_forward(*dev, slots, scale=0.125, want_lse=True)
    grads = look_attention_backward(*dev[:3], out, lse, grad_out.to(cuda_device), dev[3], slots, scale=0.125,
                                    kernel="tcgen05")
    ref_leaves = [t.double().requires_grad_(True) for t in (q, k, v, pose)]
    ref = reference_structured_look_attention(*ref_leaves, _onehot_fields(slots, 3), scale=0.125)
    ref.backward(grad_out.double())
    for got, ref_leaf in zip(grads[:4], ref_leaves):
        assert got.dtype == ref_leaf.dtype or got.dtype in (dtype, torch.float32)
        err = (got.cpu().double() - ref_leaf.grad).abs().max().item()
        assert err <= 2e-2 * max(ref_leaf.grad.abs().max().item(), 1e-3), err


def test_tensor_core_backward_agrees_with_cuda_core_backward(cuda_device):
    """Both backward implementations on the same bf16 inputs at the model's
    shape (batch 4): within the 16-bit rounding of P and dS."""
    slots, q, k, v, pose, grad_out = _slot_case(14, 14, 12, 6, 4, 3, torch.bfloat16, seed=5)
    dev = [t.to(cuda_device) for t in (q, k, v, pose)]
    out, lse = look_attention_forward(*dev, slots, scale=0.125, want_lse=True)
    go = grad_out.to(cuda_device)
    tc = look_attention_backward(*dev[:3], out, lse, go, dev[3], slots, scale=0.125, kernel="tcgen05")
    simt = look_attention_backward(*dev[:3], out, lse, go, dev[3], slots, scale=0.125, kernel="simt")
    for a, b in zip(tc[:4], simt[:4]):
        err = (a.float() - b.float()).abs().max().item()
        assert err <= 1e-2 * max(b.float().abs().max().item(), 1e-3), err


def test_probability_and_score_grad_tensors(cuda_device):
    """look_probability_score_grad (the reference's `probability` and
    `score_grad`, layers/triton_structured_look_attention.py:283-292, and the
    per-slot pose gradient) against float64 values from the same bf16 inputs."""
    from intp_preliminary_b200 import look_probability_score_grad

    slots, q, k, v, pose, grad_out = _slot_case(9, 11, 6, 3, 2, 2, torch.bfloat16, seed=9)
    n = q.shape[2]
    dev = [t.to(cuda_device) for t in (q, k, v, pose)]
    out, lse = look_attention_forward(*dev, slots, scale=0.125, want_lse=True)
    prob, sgrad, dpose = look_probability_score_grad(*dev[:3], out, lse, grad_out.to(cuda_device), dev[3], slots,
                                                     scale=0.125)
    assert prob.shape == (2, 2, n, n) and prob.dtype == torch.bfloat16
    bias = torch.zeros(2, 2, n, n, dtype=torch.float64)
    onehot = _onehot_fields(slots, 2)
    bias[:, :, 1:, 1:] = torch.einsum("bqhp,hpqk->bhqk", pose.double(), onehot)
    s = torch.einsum("bhqd,bhkd->bhqk", q.double(), k.double()) * 0.125 + bias
    p_ref = torch.softmax(s, dim=-1)
    o = out.cpu().double()
    dp = torch.einsum("bhqd,bhkd->bhqk", grad_out.double(), v.double())
    delta = (grad_out.double() * o).sum(-1, keepdim=True)
    ds_ref = p_ref * (dp - delta)
    assert (prob.cpu().double() - p_ref).abs().max().item() <= 4e-3 * p_ref.abs().max().item() + 1e-4
    assert (sgrad.cpu().double() - ds_ref).abs().max().item() <= 1e-2 * ds_ref.abs().max().item() + 1e-4
    dpose_ref = torch.einsum("bhqk,hpqk->bqhp", ds_ref[:, :, 1:, 1:], onehot)
    assert (dpose.cpu().double() - dpose_ref).abs().max().item() <= 1e-2 * dpose_ref.abs().max().item() + 1e-5


def test_fused_backward_is_deterministic(cuda_device):
    """Every gradient element of the fused tensor-core backward has one writer
    (no atomics): two runs agree bit for bit."""
    slots, q, k, v, pose, grad_out = _slot_case(14, 14, 12, 6, 4, 3, torch.bfloat16, seed=11)
    dev = [t.to(cuda_device) for t in (q, k, v, pose)]
    out, lse = look_attention_forward(*dev, slots, scale=0.125, want_lse=True)
    go = grad_out.to(cuda_device)
    a = look_attention_backward(*dev[:3], out, lse, go, dev[3], slots, scale=0.125, kernel="tcgen05")
    b = look_attention_backward(*dev[:3], out, lse, go, dev[3], slots, scale=0.125, kernel="tcgen05")
    for x, y in zip(a[:4], b[:4]):
        assert torch.equal(x, y)


def test_fused_backward_partial_needs(cuda_device):
    """Only the requested gradients: dQ and the pose gradient alone (the dK / dV
    kernel is skipped), then dV alone."""
    slots, q, k, v, pose, grad_out = _slot_case(10, 10, 8, 4, 2, 2, torch.bfloat16, seed=12)
    dev = [t.to(cuda_device) for t in (q, k, v, pose)]
    out, lse = look_attention_forward(*dev, slots, scale=0.125, want_lse=True)
    go = grad_out.to(cuda_device)
    full = look_attention_backward(*dev[:3], out, lse, go, dev[3], slots, scale=0.125, kernel="tcgen05")
    part = look_attention_backward(*dev[:3], out, lse, go, dev[3], slots, scale=0.125, kernel="tcgen05",
                                   needs=(True, False, False, True, False, False))
    assert part[1] is None and part[2] is None
    assert torch.equal(part[0], full[0]) and torch.equal(part[3], full[3])
    only_v = look_attention_backward(*dev[:3], out, lse, go, dev[3], slots, scale=0.125, kernel="tcgen05",
                                     needs=(False, False, True, False, False, False))
    assert only_v[0] is None and only_v[3] is None
    assert torch.equal(only_v[2], full[2])


def test_fused_backward_strided_qkv(cuda_device):
    """q, k, v as head-split views of one fused qkv tensor (the model's layout)
    through autograd: gradients against float64 autograd through the oracle."""
    slots = LookSlots(hexgrid.synthetic_look_slots(12, 12, 8, 4), 32)
    n = 145
    gen = torch.Generator().manual_seed(13)
    qkv = (torch.randn(2, n, 3, 3, 64, generator=gen) / 8).to(torch.bfloat16)
    pose = torch.rand(2, n - 1, 3, 32, generator=gen) * 2 - 1
    grad_out = torch.randn(2, 3, n, 64, generator=gen).to(torch.bfloat16)
    qkv_d = qkv.to(cuda_device).requires_grad_(True)
    pose_d = pose.to(cuda_device).requires_grad_(True)
    q, k, v = qkv_d.permute(2, 0, 3, 1, 4).unbind(0)
    out = structured_look_attention(q, k, v, pose_d, slots, scale=0.125)
    out.backward(grad_out.to(cuda_device))
    qkv_r = qkv.double().requires_grad_(True)
    pose_r = pose.double().requires_grad_(True)
    qr, kr, vr = qkv_r.permute(2, 0, 3, 1, 4).unbind(0)
    ref = reference_structured_look_attention(qr, kr, vr, pose_r, _onehot_fields(slots, 3), scale=0.125)
    ref.backward(grad_out.double())
    for got, want in ((qkv_d.grad, qkv_r.grad), (pose_d.grad, pose_r.grad)):
        err = (got.cpu().double() - want).abs().max().item()
        assert err <= 2e-2 * max(want.abs().max().item(), 1e-3), err


def test_tensor_core_backward_declines_other_inputs(cuda_device):
    """fp32 inputs (or dense fields) are outside the tensor-core pass: "auto"
    takes the CUDA-core backward, "tcgen05" raises."""
    slots, q, k, v, pose, grad_out = _slot_case(4, 4, 4, 2, 1, 2, torch.float32, seed=3)
    dev = [t.to(cuda_device) for t in (q, k, v, pose)]
    out, lse = look_attention_forward(*dev, slots, scale=0.125, want_lse=True)
    go = grad_out.to(cuda_device)
    grads = look_attention_backward(*dev[:3], out, lse, go, dev[3], slots, scale=0.125)
    assert grads[0].dtype == torch.float32
    with pytest.raises(ValueError):
        look_attention_backward(*dev[:3], out, lse, go, dev[3], slots, scale=0.125, kernel="tcgen05")


@pytest.mark.parametrize("seq", [130, 300])
def test_tensor_core_backward_without_look_bias(cuda_device, seq):
    """The tensor-core backward's no-bias form (SLA_BIAS_NONE through the C ABI:
    plain softmax attention, keys past the sequence masked) against float64
    autograd; the forward's LSE comes from the same C call with the same
    arguments.  Ragged query / key tiles at both lengths."""
    import ctypes

    from intp_preliminary_b200 import _lib
    from intp_preliminary_b200.look_attention import _forward_args, _stride4

    gen = torch.Generator().manual_seed(seq)
    b, h = 2, 3
    q, k, v = ((torch.randn(b, h, seq, 64, generator=gen) / 8).to(torch.bfloat16) for _ in range(3))
    grad_out = torch.randn(b, h, seq, 64, generator=gen).to(torch.bfloat16)
    slots = LookSlots(np.full((seq - 1, seq - 1), hexgrid.SLOT_NONE, dtype=np.uint8), 1)
    pose = torch.zeros(b, seq - 1, h, 1)
    dq_, dk_, dv_, go, pz = (t.to(cuda_device) for t in (q, k, v, grad_out, pose))
    out = torch.empty_like(dq_)
    lse = torch.empty(b, h, seq, device=cuda_device)
    args, keep = _forward_args(dq_, dk_, dv_, pz, slots, 0.125, None, out, lse, "tcgen05")
    args.bias_mode = _lib.SLA_BIAS_NONE
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    _lib.check(lib.sla_forward(ctypes.byref(args), stream), "forward")
    f32 = dict(dtype=torch.float32, device=cuda_device)
    grads = [torch.empty(b, h, seq, 64, **f32) for _ in range(3)]
    delta = torch.empty(b, h, seq, **f32)
    bwd = _lib.SlaBackwardArgs()
    bwd.fwd = args
    bwd.grad_out, bwd.grad_out_stride = go.data_ptr(), _stride4(go)
    bwd.grad_q, bwd.grad_k, bwd.grad_v = (g.data_ptr() for g in grads)
    bwd.grad_pose = bwd.grad_fields = bwd.grad_dense = None
    bwd.delta = delta.data_ptr()
    bwd.slots_packed_t = slots.device_packed_t(cuda_device).data_ptr()
    _lib.check(lib.sla_backward(ctypes.byref(bwd), stream), "backward")
    check_device_status(cuda_device)
    del keep
    leaves = [t.double().requires_grad_(True) for t in (q, k, v)]
    ref = torch.softmax(leaves[0] @ leaves[1].transpose(-1, -2) * 0.125, dim=-1) @ leaves[2]
    ref.backward(grad_out.double())
    assert (out.cpu().double() - ref.detach()).abs().max().item() <= 2e-2 * ref.abs().max().item()
    for got, leaf in zip(grads, leaves):
        err = (got.cpu().double() - leaf.grad).abs().max().item()
        assert err <= 2e-2 * max(leaf.grad.abs().max().item(), 1e-3), err
