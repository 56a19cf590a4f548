"""The C-ABI library loads, exports every declared symbol and its host-only
functions behave (no GPU needed: nothing here launches a kernel)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import _lib
from intp_preliminary_b200.look_attention import LookSlots

HEADER = Path(__file__).resolve().parent.parent / "include" / "intp_b200.h"
SVIT_HEADER = HEADER.with_name("intp_share_vit.h")


def _declared_functions(header=HEADER):
    text = header.read_text()
    return sorted(set(re.findall(r"INTP_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    for header, expected in ((HEADER, _lib.EXPORTED_SYMBOLS), (SVIT_HEADER, _lib.SHARE_VIT_SYMBOLS)):
        declared = _declared_functions(header)
        assert declared, f"no declarations found in {header.name}"
        assert set(declared) == set(expected)
        for name in declared:
            assert hasattr(lib, name), name
    headers = sorted(p.name for p in HEADER.parent.glob("*.h"))
    assert headers == ["intp_b200.h", "intp_share_vit.h"]


def test_svit_struct_layout_matches_header_field_order():
    text = SVIT_HEADER.read_text()
    body = text[text.index("typedef struct svit_embed_args"):text.index("} svit_embed_args;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    names = re.findall(r"(\w+)\s*[;,]", body)
    assert names == [f[0] for f in _lib.SvitEmbedArgs._fields_]
    body = text[text.index("typedef struct svit_gather_plan"):text.index("} svit_gather_plan;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    assert re.findall(r"(\w+)\s*[;,]", body) == [f[0] for f in _lib.SvitGatherPlan._fields_]


def test_svit_host_side_argument_checks():
    lib = _lib.load()
    # zero-sized work is a no-op; bad sizes are rejected before any launch
    assert lib.svit_gather_patches(None, 0, 0, None, None, 0, 0, None, None) == _lib.INTP_OK
    assert lib.svit_gather_patches(None, -1, 0, None, None, 1, 8, None, None) == _lib.INTP_ERR_ARGUMENT
    plan = _lib.SvitGatherPlan(16, 16, 16, 2, 8, 100)
    assert lib.svit_gather_patches_staged(None, 0, 0, ctypes.byref(plan), None, 0, 0, None, None) == _lib.INTP_OK
    assert lib.svit_gather_patches_staged(None, 1, 10, None, None, 9, 8, None, None) == _lib.INTP_ERR_ARGUMENT
    fake = 1 << 20  # never dereferenced: every case below is rejected before a launch
    plan.groups = 3  # 9 patches in groups of 8 are 2 groups
    assert lib.svit_gather_patches_staged(fake, 1, 10, ctypes.byref(plan), fake, 9, 8, fake, None) == \
        _lib.INTP_ERR_ARGUMENT
    plan.groups, plan.local_index = 2, 18  # local_index not 16-byte aligned
    assert lib.svit_gather_patches_staged(fake, 1, 10, ctypes.byref(plan), fake, 9, 8, fake, None) == \
        _lib.INTP_ERR_LAYOUT
    plan.local_index = 16  # images of 10 floats are not whole 16-byte units
    assert lib.svit_gather_patches_staged(fake, 1, 10, ctypes.byref(plan), fake, 9, 8, fake, None) == \
        _lib.INTP_ERR_LAYOUT
    plan.max_stage = 15000  # 240 KB of shared memory
    assert lib.svit_gather_patches_staged(fake, 1, 12, ctypes.byref(plan), fake, 9, 8, fake, None) == \
        _lib.INTP_ERR_UNSUPPORTED
    assert lib.svit_add_layernorm(None, 0, None, 0, None, None, 1e-6, 0, 192, None, 0, None) == _lib.INTP_OK
    assert lib.svit_add_layernorm(None, 0, None, 0, None, None, 1e-6, 3, 192, None, 0, None) == _lib.INTP_ERR_ARGUMENT
    a = _lib.SvitEmbedArgs()
    a.batch, a.patches, a.bases, a.directions, a.look_heads, a.look_poses, a.slots = 1, 4, 96, 6, 36, 12, 200
    assert lib.svit_embed_post(ctypes.byref(a), None) == _lib.INTP_ERR_SHAPE


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.intp_abi_version() == 3
    assert _lib.status_string(_lib.INTP_OK) == "ok"
    assert "timed out" in _lib.status_string(_lib.INTP_ERR_TIMEOUT)


def test_backward_struct_layout_matches_header_field_order():
    text = HEADER.read_text()
    body = text[text.index("typedef struct sla_backward_args"):text.index("} sla_backward_args;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    names = re.findall(r"(\w+)(?:\[4\])?\s*[;,]", body)
    assert names == [f[0] for f in _lib.SlaBackwardArgs._fields_]


def test_struct_layout_matches_header_field_order():
    text = HEADER.read_text()
    body = text[text.index("typedef struct sla_forward_args"):text.index("} sla_forward_args;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    names = re.findall(r"(\w+)(?:\[4\])?\s*[;,]", body)
    ctypes_names = [f[0] for f in _lib.SlaForwardArgs._fields_]
    assert names == ctypes_names


def test_slot_table_bytes():
    lib = _lib.load()
    pb, fb = ctypes.c_int64(), ctypes.c_int64()
    assert lib.sla_slot_table_bytes(197, ctypes.byref(pb), ctypes.byref(fb)) == 0
    assert pb.value == 2 * 4 * 8192 and fb.value == 8
    assert lib.sla_slot_table_bytes(0, ctypes.byref(pb), ctypes.byref(fb)) == _lib.INTP_ERR_ARGUMENT


def test_pack_slot_table_layout():
    rng = np.random.default_rng(0)
    patches = 150
    table = rng.integers(0, 20, size=(patches, patches)).astype(np.uint8)
    table[rng.random((patches, patches)) < 0.5] = 255
    packed, flags = LookSlots(table, 20).host_packed()
    seq = patches + 1
    nkt = (seq + 63) // 64
    for i in range(seq):
        for j in range(0, seq, 7):
            qt, r = divmod(i, 128)
            kt, c = divmod(j, 64)
            value = packed[(qt * nkt + kt) * 8192 + (c // 16) * 2048 + r * 16 + c % 16]
            if i == 0 or j == 0 or table[i - 1, j - 1] == 255:
                assert value == 20
            else:
                assert value == table[i - 1, j - 1]
    assert flags.sum() > 0
    # keys past the sequence end carry n_slots + 1 (masked); their tile is flagged
    for qt in range((seq + 127) // 128):
        kt = nkt - 1
        for c in range(seq % 64, 64):
            for r in (0, 77, 127):
                assert packed[(qt * nkt + kt) * 8192 + (c // 16) * 2048 + r * 16 + c % 16] == 21
        assert flags[qt * nkt + kt] == 0xF


def test_pack_rejects_out_of_range_slot():
    table = np.full((4, 4), 255, np.uint8)
    table[1, 2] = 7
    with pytest.raises(ValueError):
        LookSlots(table, 5)


def test_forward_rejects_bad_arguments_without_launching():
    lib = _lib.load()
    args = _lib.SlaForwardArgs()
    args.batch, args.heads, args.seq, args.head_dim = 1, 1, 0, 64
    assert lib.sla_forward(ctypes.byref(args), None) == _lib.INTP_ERR_SHAPE
    args.seq, args.dtype = 8, 9
    assert lib.sla_forward(ctypes.byref(args), None) == _lib.INTP_ERR_DTYPE
    args.dtype = _lib.INTP_BF16
    assert lib.sla_forward(ctypes.byref(args), None) == _lib.INTP_ERR_ARGUMENT  # null pointers
    assert lib.sla_forward(None, None) == _lib.INTP_ERR_ARGUMENT
    assert lib.nl1_forward(None, None, None, -1, 1, 1, None) == _lib.INTP_ERR_SHAPE


def test_operators_refuse_cpu_tensors():
    import torch

    from intp_preliminary_b200 import negative_l1_distance, structured_look_attention

    q = torch.randn(1, 1, 3, 16)
    with pytest.raises(ValueError, match="CUDA"):
        structured_look_attention(q, q, q, torch.randn(1, 2, 1, 4), torch.randn(1, 4, 2, 2), scale=0.25)
    with pytest.raises(ValueError, match="CUDA"):
        negative_l1_distance(torch.randn(3, 4), torch.randn(2, 4))
    with pytest.raises(ValueError, match="feature"):
        negative_l1_distance(torch.randn(3, 4), torch.randn(2, 5))


def test_slot_fields_dense_expansion_matches_oracle():
    """LookSlotFields.dense() (host tensors) equals the oracle's expansion."""
    from intp_preliminary_b200 import LookSlotFields
    from oracle.look_attention import slot_fields_dense_np

    rng = np.random.default_rng(4)
    table = rng.integers(0, 9, size=(11, 11)).astype(np.uint8)
    table[rng.random((11, 11)) < 0.3] = 255
    values = torch.from_numpy(rng.standard_normal((2, 3, 9)).astype(np.float32))
    look = LookSlotFields(LookSlots(table, 9), values)
    assert look.shape == (2, 3, 11, 11)
    np.testing.assert_array_equal(look.dense().numpy(), slot_fields_dense_np(values.numpy(), table))
    with pytest.raises(ValueError):
        LookSlotFields(LookSlots(table, 9), values[:, :, :8])


def test_slot_fields_mode_argument_checks():
    """SLOT_FIELDS needs pose, slot values, the packed table and a slot count."""
    lib = _lib.load()
    args = _lib.SlaForwardArgs()
    args.batch, args.heads, args.seq, args.head_dim = 1, 1, 5, 64
    args.dtype = _lib.INTP_BF16
    for name in ("q", "k", "v", "out"):
        setattr(args, name, 16)
        setattr(args, name + "_stride", _lib._Stride(320, 320, 64, 1))
    args.bias_mode = _lib.SLA_BIAS_SLOT_FIELDS
    args.poses = 12
    args.pose = 16
    args.slots_packed = args.slot_tile_flags = 16
    args.slots = 8
    assert lib.sla_forward(ctypes.byref(args), None) == _lib.INTP_ERR_ARGUMENT  # no slot values
    args.fields = 16
    args.slots = 0
    assert lib.sla_forward(ctypes.byref(args), None) == _lib.INTP_ERR_ARGUMENT  # no slots
