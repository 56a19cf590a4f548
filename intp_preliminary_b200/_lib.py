"""ctypes binding of ``libintp_b200.so`` (the C ABI in ``include/intp_b200.h``).

The shared library is the only compute path of this package: if it is missing
or cannot be loaded, every operator raises instead of falling back to CPU or
PyTorch code.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libintp_b200.so"

INTP_OK = 0
INTP_ERR_ARGUMENT = 1
INTP_ERR_SHAPE = 2
INTP_ERR_DTYPE = 3
INTP_ERR_LAYOUT = 4
INTP_ERR_ARCH = 5
INTP_ERR_LAUNCH = 6
INTP_ERR_TIMEOUT = 7
INTP_ERR_UNSUPPORTED = 8

INTP_F32, INTP_F16, INTP_BF16 = 0, 1, 2
SLA_BIAS_NONE, SLA_BIAS_FIELDS, SLA_BIAS_SLOTS, SLA_BIAS_SLOT_FIELDS = 0, 1, 2, 3
SLA_SLOT_NONE = 255
ABI_VERSION = 3
SLA_KERNEL_AUTO, SLA_KERNEL_SIMT, SLA_KERNEL_TCGEN05 = 0, 1, 2

# Every symbol include/intp_b200.h declares.
EXPORTED_SYMBOLS = (
    "sla_forward",
    "sla_backward",
    "sla_probability_score_grad",
    "sla_slot_table_bytes",
    "sla_pack_slot_table",
    "nl1_forward",
    "nl1_backward",
    "sla_read_status",
    "sla_forward_noalloc",
    "dlg_forward",
    "dlg_backward",
    "intp_set_wait_budget_ns",
    "intp_device_info",
    "intp_abi_version",
    "intp_status_string",
)
# Every symbol include/intp_share_vit.h declares.
SHARE_VIT_SYMBOLS = (
    "svit_gather_patches",
    "svit_gather_patches_staged",
    "svit_embed_post",
    "svit_tokenizer_gemm",
    "svit_add_layernorm",
    "svit_linear_gelu",
    "svit_linear_bias",
    "svit_linear_residual_layernorm",
)

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_vp = ctypes.c_void_p
_Stride = _i64 * 4


class SlaForwardArgs(ctypes.Structure):
    """Mirror of ``sla_forward_args`` (field order and types must match)."""

    _fields_ = [
        ("batch", _i64), ("heads", _i64), ("seq", _i64), ("head_dim", _i64),
        ("scale", ctypes.c_float),
        ("dtype", _i32),
        ("q", _vp), ("q_stride", _Stride),
        ("k", _vp), ("k_stride", _Stride),
        ("v", _vp), ("v_stride", _Stride),
        ("out", _vp), ("out_stride", _Stride),
        ("lse", _vp),
        ("bias_mode", _i32),
        ("poses", _i64),
        ("pose", _vp), ("pose_stride", _Stride), ("pose_dtype", _i32),
        ("fields", _vp), ("fields_stride", _Stride), ("fields_dtype", _i32),
        ("slots_packed", _vp),
        ("slot_tile_flags", _vp),
        ("dense", _vp), ("dense_stride", _Stride), ("dense_dtype", _i32),
        ("status", _vp),
        ("kernel", _i32),
        ("slots", _i64),
    ]


class SlaBackwardArgs(ctypes.Structure):
    """Mirror of ``sla_backward_args`` (field order and types must match)."""

    _fields_ = [
        ("fwd", SlaForwardArgs),
        ("grad_out", _vp), ("grad_out_stride", _Stride),
        ("grad_q", _vp), ("grad_k", _vp), ("grad_v", _vp),
        ("grad_pose", _vp),
        ("grad_fields", _vp),
        ("grad_dense", _vp),
        ("delta", _vp),
        ("slots_packed_t", _vp),
    ]


class SlaProbabilityScoreGradArgs(ctypes.Structure):
    """Mirror of ``sla_probability_score_grad_args`` (field order and types must match)."""

    _fields_ = [
        ("fwd", SlaForwardArgs),
        ("grad_out", _vp), ("grad_out_stride", _Stride),
        ("probability", _vp), ("score_grad", _vp),
        ("ld", _i64),
        ("grad_pose", _vp),
    ]


class SvitEmbedArgs(ctypes.Structure):
    """Mirror of ``svit_embed_args`` (include/intp_share_vit.h)."""

    _fields_ = [
        ("batch", _i64), ("patches", _i64),
        ("bases", _i32), ("directions", _i32),
        ("look_heads", _i32), ("look_poses", _i32),
        ("slots", _i32),
        ("resp", _vp), ("resp_stride", _i64),
        ("token_null", _vp), ("direction_coef", _vp), ("output_bias", _vp),
        ("cls", _vp), ("pos_embed", _vp), ("look_null", _vp), ("slot_fields", _vp),
        ("x", _vp), ("values", _vp),
        ("look_pose", _vp),
    ]


class DlgArgs(ctypes.Structure):
    """Mirror of ``dlg_args`` (include/intp_b200.h)."""

    _fields_ = [
        ("batch", _i64), ("queries", _i64), ("heads", _i64),
        ("dtype", _i32),
        ("grid", _vp), ("grid_stride", _i64 * 5),
        ("radial0", _vp), ("radial1", _vp), ("angular0", _vp), ("angular1", _vp),
        ("radial_fraction", _vp), ("angular_fraction", _vp), ("valid", _vp),
        ("table_stride", (_i64 * 2) * 7),
        ("out", _vp), ("out_stride", _Stride),
    ]


class DlgGradStrides(ctypes.Structure):
    """Mirror of ``dlg_grad_strides`` (include/intp_b200.h)."""

    _fields_ = [("stride", _Stride)]


class SvitGatherPlan(ctypes.Structure):
    """Mirror of ``svit_gather_plan`` (include/intp_share_vit.h)."""

    _fields_ = [
        ("stage_offset", _vp), ("stage_begin", _vp), ("local_index", _vp),
        ("groups", _i64), ("group_patches", _i64), ("max_stage", _i64),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeLibraryError(RuntimeError):
    """The CUDA extension is missing or does not export the expected ABI."""


def load() -> ctypes.CDLL:
    """Load the library once; raise NativeLibraryError when it is unavailable."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise NativeLibraryError(
                f"{LIB_PATH} is not built; run `python -m intp_preliminary_b200.build`"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        missing = [name for name in EXPORTED_SYMBOLS + SHARE_VIT_SYMBOLS if not hasattr(lib, name)]
        if missing:
            raise NativeLibraryError(f"{LIB_PATH} lacks symbols {missing}")
        lib.sla_forward.argtypes = [ctypes.POINTER(SlaForwardArgs), _vp]
        lib.sla_forward.restype = _i32
        lib.sla_backward.argtypes = [ctypes.POINTER(SlaBackwardArgs), _vp]
        lib.sla_backward.restype = _i32
        lib.sla_probability_score_grad.argtypes = [ctypes.POINTER(SlaProbabilityScoreGradArgs), _vp]
        lib.sla_probability_score_grad.restype = _i32
        lib.nl1_backward.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]
        lib.nl1_backward.restype = _i32
        lib.sla_slot_table_bytes.argtypes = [_i64, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]
        lib.sla_slot_table_bytes.restype = _i32
        lib.sla_pack_slot_table.argtypes = [_vp, _i64, _i32, _vp, _vp]
        lib.sla_pack_slot_table.restype = _i32
        lib.nl1_forward.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _vp]
        lib.nl1_forward.restype = _i32
        lib.sla_forward_noalloc.argtypes = [ctypes.POINTER(SlaForwardArgs), _vp, _vp]
        lib.sla_forward_noalloc.restype = _i32
        lib.dlg_forward.argtypes = [ctypes.POINTER(DlgArgs), _vp]
        lib.dlg_forward.restype = _i32
        lib.dlg_backward.argtypes = [ctypes.POINTER(DlgArgs), _vp, ctypes.POINTER(DlgGradStrides), _vp, _vp]
        lib.dlg_backward.restype = _i32
        lib.sla_read_status.argtypes = [_vp, ctypes.POINTER(_i32), _vp]
        lib.sla_read_status.restype = _i32
        lib.intp_set_wait_budget_ns.argtypes = [ctypes.c_uint64]
        lib.intp_set_wait_budget_ns.restype = _i32
        lib.intp_device_info.argtypes = [ctypes.POINTER(_i32)] * 3
        lib.intp_device_info.restype = _i32
        lib.svit_gather_patches.argtypes = [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _vp]
        lib.svit_gather_patches.restype = _i32
        lib.svit_gather_patches_staged.argtypes = [_vp, _i64, _i64, ctypes.POINTER(SvitGatherPlan), _vp, _i64, _i64,
                                                   _vp, _vp]
        lib.svit_gather_patches_staged.restype = _i32
        lib.svit_embed_post.argtypes = [ctypes.POINTER(SvitEmbedArgs), _vp]
        lib.svit_embed_post.restype = _i32
        lib.svit_tokenizer_gemm.argtypes = [ctypes.POINTER(SvitEmbedArgs), _vp, _i64, _i32, _vp, _vp, _vp]
        lib.svit_tokenizer_gemm.restype = _i32
        lib.svit_add_layernorm.argtypes = [_vp, _i64, _vp, _i64, _vp, _vp, ctypes.c_float, _i64, _i64, _vp, _i64, _vp]
        lib.svit_add_layernorm.restype = _i32
        lib.svit_linear_gelu.argtypes = [_vp, _i64, _i64, _i32, _vp, _vp, _i32, _vp, _i64, _vp, _vp]
        lib.svit_linear_gelu.restype = _i32
        lib.svit_linear_bias.argtypes = [_vp, _i64, _i64, _i32, _vp, _vp, _i32, _vp, _i64, _vp, _vp]
        lib.svit_linear_bias.restype = _i32
        lib.svit_linear_residual_layernorm.argtypes = [_vp, _i64, _i64, _i32, _vp, _vp, _i32, _vp, _i64, _vp, _vp,
                                                       ctypes.c_float, _vp, _i64, _vp, _vp]
        lib.svit_linear_residual_layernorm.restype = _i32
        lib.intp_abi_version.argtypes = []
        lib.intp_abi_version.restype = _i32
        lib.intp_status_string.argtypes = [_i32]
        lib.intp_status_string.restype = ctypes.c_char_p
        if lib.intp_abi_version() != ABI_VERSION:
            raise NativeLibraryError("libintp_b200.so ABI version mismatch")
        _lib = lib
        return lib


def status_string(status: int) -> str:
    return load().intp_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    """Raise the error the reference would raise for a failed launch."""
    if status == INTP_OK:
        return
    message = f"{what}: {status_string(status)} (status {status})"
    if status in (INTP_ERR_ARGUMENT, INTP_ERR_SHAPE, INTP_ERR_DTYPE, INTP_ERR_LAYOUT):
        raise ValueError(message)
    raise RuntimeError(message)
