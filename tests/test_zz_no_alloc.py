"""The allocation-free Look-attention entry point (sla_forward_noalloc).

Some callers of this library cannot allocate device memory when they run the
attention: plugins whose enqueue step must not allocate because the host
framework plans every buffer ahead of time, serving loops that forbid
allocation after start-up, and callers with a fixed device-memory budget.
sla_forward_noalloc lets them pass only their inputs and outputs (the plain
slot table included); the library packs the table into scratch memory it owns
as a file-scope __device__ array.

These tests call that entry point through the C ABI and compare its output
with the regular sla_forward path (packed table built on the host), on calls
in a row with different lattices so that stale scratch contents would show.
The file is named to be collected last; it also passes on its own in a fresh
process.
"""

import ctypes

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import LookSlots, _lib, hexgrid, look_attention_forward

pytestmark = pytest.mark.gpu
TOL = 8e-3  # the bf16 tensor-core tolerance used by the other Look-attention tests


def _inputs(batch, heads, rows, cols, n_dir, device, seed):
    g = torch.Generator().manual_seed(seed)
    patches = rows * cols
    q, k, v = ((torch.randn(batch, heads, patches + 1, 64, generator=g) / 8).to(torch.bfloat16) for _ in range(3))
    pose = torch.rand(batch, patches, heads, n_dir * 4, generator=g) * 2 - 1
    slots = hexgrid.synthetic_look_slots(rows, cols, n_dir, 4)
    return [t.to(device) for t in (q, k, v, pose)], slots


def _noalloc_call(q, k, v, pose, slots_dev, n_slots, out, status=None):
    """One sla_forward_noalloc call through ctypes; returns the status code."""
    args = _lib.SlaForwardArgs()
    args.batch, args.heads, args.seq, args.head_dim = q.shape
    args.scale = 0.125
    args.dtype = _lib.INTP_BF16
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        setattr(args, name, t.data_ptr())
        setattr(args, name + "_stride", _lib._Stride(*t.stride()))
    args.bias_mode = _lib.SLA_BIAS_SLOTS
    args.poses = n_slots
    args.pose, args.pose_stride, args.pose_dtype = pose.data_ptr(), _lib._Stride(*pose.stride()), _lib.INTP_F32
    args.status = status.data_ptr() if status is not None else None
    lib = _lib.load()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    return lib.sla_forward_noalloc(ctypes.byref(args), ctypes.c_void_p(slots_dev.data_ptr()), ctypes.c_void_p(stream))


@pytest.mark.parametrize("order", ["small_large_small"])
def test_noalloc_matches_regular_entry_point(cuda_device, order):
    cases = [(2, 3, 14, 14, 12, 1), (2, 2, 32, 32, 8, 2), (3, 3, 14, 14, 12, 3)]
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for batch, heads, rows, cols, n_dir, seed in cases:
        (q, k, v, pose), slots = _inputs(batch, heads, rows, cols, n_dir, cuda_device, seed)
        n_slots = n_dir * 4
        slots_dev = torch.from_numpy(slots).to(cuda_device)
        out = torch.empty_like(q)
        assert _noalloc_call(q, k, v, pose, slots_dev, n_slots, out, status) == _lib.INTP_OK
        expected, _ = look_attention_forward(q, k, v, pose, LookSlots(slots, n_slots), scale=0.125, kernel="tcgen05")
        torch.cuda.synchronize(cuda_device)
        assert int(status.item()) == 0
        err = (out.float() - expected.float()).abs().max().item()
        assert err <= TOL, f"{order}: case {rows}x{cols} differs by {err}"


def test_noalloc_twice_in_a_row_without_status_word(cuda_device):
    (q, k, v, pose), slots = _inputs(2, 3, 8, 9, 12, cuda_device, 11)
    slots_dev = torch.from_numpy(slots).to(cuda_device)
    expected, _ = look_attention_forward(q, k, v, pose, LookSlots(slots, 48), scale=0.125, kernel="tcgen05")
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        assert _noalloc_call(q, k, v, pose, slots_dev, 48, out) == _lib.INTP_OK
        torch.cuda.synchronize(cuda_device)
        assert (out.float() - expected.float()).abs().max().item() <= TOL


def test_noalloc_rejects_sequences_beyond_its_scratch(cuda_device):
    rows, cols = 33, 32  # 1057 tokens > SLA_NOALLOC_MAX_SEQ = 1025
    (q, k, v, pose), slots = _inputs(1, 1, rows, cols, 8, cuda_device, 5)
    out = torch.zeros_like(q)
    slots_dev = torch.from_numpy(slots).to(cuda_device)
    assert _noalloc_call(q, k, v, pose, slots_dev, 32, out) == _lib.INTP_ERR_UNSUPPORTED
    torch.cuda.synchronize(cuda_device)
    assert (out == 0).all()


def test_noalloc_rejects_bad_arguments_without_launching(cuda_device):
    """The host-side checks of sla_forward run first: null tensors, bad dtype
    codes and a bad kernel selector return an error and write nothing."""
    (q, k, v, pose), slots = _inputs(1, 2, 6, 6, 12, cuda_device, 7)
    slots_dev = torch.from_numpy(slots).to(cuda_device)
    out = torch.zeros_like(q)
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)

    def call(**override):
        args = _lib.SlaForwardArgs()
        args.batch, args.heads, args.seq, args.head_dim = q.shape
        args.scale, args.dtype = 0.125, _lib.INTP_BF16
        for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
            setattr(args, name, t.data_ptr())
            setattr(args, name + "_stride", _lib._Stride(*t.stride()))
        args.bias_mode, args.poses = _lib.SLA_BIAS_SLOTS, 48
        args.pose, args.pose_stride, args.pose_dtype = pose.data_ptr(), _lib._Stride(*pose.stride()), _lib.INTP_F32
        for key, value in override.items():
            setattr(args, key, value)
        return lib.sla_forward_noalloc(ctypes.byref(args), ctypes.c_void_p(slots_dev.data_ptr()), stream)

    assert call(out=None) == _lib.INTP_ERR_ARGUMENT
    assert call(q=None) == _lib.INTP_ERR_ARGUMENT
    assert call(pose=None) == _lib.INTP_ERR_ARGUMENT
    assert call(dtype=7) == _lib.INTP_ERR_DTYPE
    assert call(pose_dtype=9) == _lib.INTP_ERR_DTYPE
    assert call(kernel=5) == _lib.INTP_ERR_ARGUMENT
    assert call(kernel=_lib.SLA_KERNEL_SIMT) == _lib.INTP_ERR_UNSUPPORTED
    assert call(head_dim=0) == _lib.INTP_ERR_SHAPE
    torch.cuda.synchronize(cuda_device)
    assert (out == 0).all()


def test_noalloc_reports_out_of_range_slot_bytes(cuda_device):
    """A slot byte >= n_slots (other than 255) gets no bias, as a table packed
    on the host would refuse it; the caller's status word reports it."""
    (q, k, v, pose), slots = _inputs(1, 2, 6, 6, 12, cuda_device, 9)
    bad = slots.copy()
    bad[3, 4] = 60  # n_slots = 48
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = torch.empty_like(q)
    assert _noalloc_call(q, k, v, pose, torch.from_numpy(bad).to(cuda_device), 48, out, status) == _lib.INTP_OK
    code = ctypes.c_int32()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    rc = _lib.load().sla_read_status(ctypes.c_void_p(status.data_ptr()), ctypes.byref(code), stream)
    assert rc == _lib.INTP_ERR_ARGUMENT and code.value == 0x201
    assert int(status.item()) == 0  # read and cleared
    fixed = slots.copy()
    fixed[3, 4] = _lib.SLA_SLOT_NONE
    expected, _ = look_attention_forward(q, k, v, pose, LookSlots(fixed, 48), scale=0.125, kernel="tcgen05")
    assert (out.float() - expected.float()).abs().max().item() <= TOL


def test_noalloc_call_leaves_device_memory_unchanged(cuda_device):
    """After the first call on the device (its one-time set-up), a call changes
    neither PyTorch's allocation count nor the device's free memory."""
    (q, k, v, pose), slots = _inputs(2, 3, 14, 14, 12, cuda_device, 13)
    slots_dev = torch.from_numpy(slots).to(cuda_device)
    out = torch.empty_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    assert _noalloc_call(q, k, v, pose, slots_dev, 48, out, status) == _lib.INTP_OK
    torch.cuda.synchronize(cuda_device)
    allocated = torch.cuda.memory_allocated(cuda_device)
    free_before, _ = torch.cuda.mem_get_info(cuda_device)
    for _ in range(3):
        assert _noalloc_call(q, k, v, pose, slots_dev, 48, out, status) == _lib.INTP_OK
    torch.cuda.synchronize(cuda_device)
    free_after, _ = torch.cuda.mem_get_info(cuda_device)
    assert torch.cuda.memory_allocated(cuda_device) == allocated
    assert free_after == free_before
    assert int(status.item()) == 0
