"""The bounded-wait unwind of the tensor-core Look-attention kernels, made to run
out on purpose without a hung wait.

Every mbarrier wait of the tensor-core kernels gives up after a wall-clock
budget (one second by default).  ``intp_set_wait_budget_ns`` shortens the
budget of the pipeline waits to a few hundred nanoseconds - far below the
latency of the first tensor-map load - so the first wait that cannot be met at
once runs out: that role raises the CTA's abort flag, every role stops, the
producer and MMA warps drain their in-flight copies and MMAs under the full
budget, tensor memory is freed and the status word records the role's code.
The host must see the error through ``check_device_status`` and the very next
launch with the default budget must succeed and match the oracle (the context
stays usable).
"""

import ctypes

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import LookSlots, _lib, check_device_status, hexgrid, look_attention_forward
from oracle.look_attention import slot_look_attention_np

pytestmark = pytest.mark.gpu


def _inputs(rows, cols, device, seed):
    g = torch.Generator().manual_seed(seed)
    seq = rows * cols + 1
    q, k, v = ((torch.randn(4, 3, seq, 64, generator=g) / 8).to(torch.bfloat16).to(device) for _ in range(3))
    pose = (torch.rand(4, seq - 1, 3, 48, generator=g) * 2 - 1).to(device)
    return q, k, v, pose, hexgrid.synthetic_look_slots(rows, cols, 12, 4)


@pytest.mark.parametrize("rows,cols", [(14, 14), (24, 24)])  # the single-pass (N <= 256) and the tiled kernel
def test_short_budget_reports_timeout_and_next_call_is_clean(cuda_device, rows, cols):
    lib = _lib.load()
    q, k, v, pose, slots = _inputs(rows, cols, cuda_device, rows)
    look = LookSlots(slots, 48)
    check_device_status(cuda_device)  # start from a clean status word
    assert lib.intp_set_wait_budget_ns(ctypes.c_uint64(300)) == _lib.INTP_OK
    try:
        look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="tcgen05")
        with pytest.raises(RuntimeError, match="device wait failed: code 0x10"):
            check_device_status(cuda_device)
    finally:
        assert lib.intp_set_wait_budget_ns(ctypes.c_uint64(1_000_000_000)) == _lib.INTP_OK
    out, _ = look_attention_forward(q, k, v, pose, look, scale=0.125, kernel="tcgen05")
    check_device_status(cuda_device)
    for b, h in ((0, 0), (3, 2)):
        exact = slot_look_attention_np(q[b:b + 1, h:h + 1].float().cpu().numpy(),
                                       k[b:b + 1, h:h + 1].float().cpu().numpy(),
                                       v[b:b + 1, h:h + 1].float().cpu().numpy(),
                                       pose[b:b + 1, :, h:h + 1].cpu().numpy(), slots, scale=0.125)
        assert np.abs(out[b:b + 1, h:h + 1].float().cpu().numpy() - exact).max() <= 8e-3


def test_wait_budget_argument_checks():
    lib = _lib.load()
    assert lib.intp_set_wait_budget_ns(ctypes.c_uint64(0)) == _lib.INTP_ERR_ARGUMENT
    assert lib.intp_set_wait_budget_ns(ctypes.c_uint64(2_000_000_000)) == _lib.INTP_ERR_ARGUMENT
