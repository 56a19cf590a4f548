"""Structured Look attention on B200: the drop-in for
``layers/triton_structured_look_attention.py`` of the reference.

``structured_look_attention(q, k, v, pose, fields, *, scale, dense_bias=None)``
keeps the reference signature and result (layers/triton_structured_look_attention.py:412-424):

    S = scale * q @ k^T                         (B, H, N, N), fp32
    S[:, :, 1:, 1:] += einsum("bqhp,hpqk->bhqk", pose, fields) (+ dense_bias)
    out = softmax(S, -1) @ v                    cast to q.dtype

with ``q/k/v`` of shape ``(B, H, N, D)`` (token 0 is CLS, N = Np + 1), ``pose``
``(B, Np, H, P)`` and ``fields`` ``(H, P, Np, Np)``.

``fields`` may also be a :class:`LookSlots`, the compact form of one-hot fields
(``fields[h, p, q, k] = 1[slot(q, k) == p]``): the per-pair slot table is
shared by every batch and head and the bias becomes ``pose[b, q, h, slot]``.
That is the form the tensor-core kernel consumes without ever materialising an
``Np x Np`` bias or field tensor.

``fields`` may also be a :class:`LookSlotFields`: fields whose every
``(Np, Np)`` plane is a per-slot value gathered by such a pair table
(``fields[h, p, q, k] = values[h, p, slot(q, k)]``), which is how the
reference model's Look bank builds them (model/deit_tiny_rot_hex_look.py:397-451).
The bias is then ``sum_p pose[b, q, h, p] * values[h, p, slot(q, k)]``, formed per
query inside the kernel from the P pose values and the ``(H, P, S)`` slot values.

Every call runs the CUDA kernels of ``libintp_b200.so``; there is no CPU or
PyTorch fallback.  CPU tensors raise ``ValueError`` like any other input the
kernels cannot take.
"""

from __future__ import annotations

import ctypes
import threading

import numpy as np
import torch

from . import _lib

_DTYPE_CODE = {torch.float32: _lib.INTP_F32, torch.float16: _lib.INTP_F16, torch.bfloat16: _lib.INTP_BF16}
_KERNELS = {"auto": _lib.SLA_KERNEL_AUTO, "simt": _lib.SLA_KERNEL_SIMT, "tcgen05": _lib.SLA_KERNEL_TCGEN05}


class LookSlots:
    """Pair table standing in for one-hot Look fields of shape ``(H, P, Np, Np)``.

    ``slots`` is an ``(Np, Np)`` uint8 array/tensor: ``slots[q, k]`` is the
    index ``p < n_slots`` of the query's Look field that pair ``(q, k)`` reads,
    or 255 for "no bias".  The packed tile layout the kernels read is built
    once on the host (``sla_pack_slot_table``) and cached per device.
    """

    def __init__(self, slots, n_slots: int, heads: int | None = None) -> None:
        table = slots.detach().cpu().numpy() if isinstance(slots, torch.Tensor) else np.asarray(slots)
        if table.ndim != 2 or table.shape[0] != table.shape[1]:
            raise ValueError("slots must be a square (Np, Np) table")
        if not 1 <= int(n_slots) <= 253:
            raise ValueError("n_slots must be in [1, 253]")
        table = np.ascontiguousarray(table.astype(np.uint8))
        used = table[table != _lib.SLA_SLOT_NONE]
        if used.size and int(used.max()) >= int(n_slots):
            raise ValueError("slot index out of range for n_slots")
        self.table = table
        self.n_slots = int(n_slots)
        self.heads = heads
        self._packed: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self._host: tuple[np.ndarray, np.ndarray] | None = None
        self._packed_t: dict[int, torch.Tensor] = {}
        self._host_t: np.ndarray | None = None
        self._lock = threading.Lock()

    @property
    def patch_count(self) -> int:
        return int(self.table.shape[0])

    @property
    def shape(self) -> tuple[int, ...]:
        heads = -1 if self.heads is None else self.heads
        return (heads, self.n_slots, self.patch_count, self.patch_count)

    def host_packed(self) -> tuple[np.ndarray, np.ndarray]:
        """Packed tiles and per-tile flags as host arrays (pure CPU)."""
        if self._host is None:
            lib = _lib.load()
            seq = self.patch_count + 1
            pb, fb = ctypes.c_int64(), ctypes.c_int64()
            _lib.check(lib.sla_slot_table_bytes(seq, ctypes.byref(pb), ctypes.byref(fb)), "sla_slot_table_bytes")
            packed = np.empty(pb.value, dtype=np.uint8)
            flags = np.empty(fb.value, dtype=np.uint8)
            _lib.check(
                lib.sla_pack_slot_table(
                    self.table.ctypes.data, self.patch_count, self.n_slots, packed.ctypes.data, flags.ctypes.data
                ),
                "sla_pack_slot_table",
            )
            self._host = (packed, flags)
        return self._host

    def host_packed_t(self) -> np.ndarray:
        """Packed tiles of the transposed table (``[k, q]``), read by the key-major
        backward kernel (pure CPU)."""
        if self._host_t is None:
            lib = _lib.load()
            packed, flags = (np.empty_like(x) for x in self.host_packed())
            table_t = np.ascontiguousarray(self.table.T)
            _lib.check(
                lib.sla_pack_slot_table(
                    table_t.ctypes.data, self.patch_count, self.n_slots, packed.ctypes.data, flags.ctypes.data
                ),
                "sla_pack_slot_table",
            )
            self._host_t = packed
        return self._host_t

    def device_packed_t(self, device: torch.device) -> torch.Tensor:
        index = torch.device(device).index
        with self._lock:
            if index not in self._packed_t:
                self._packed_t[index] = torch.from_numpy(self.host_packed_t()).to(device)
            return self._packed_t[index]

    def device_packed(self, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        index = torch.device(device).index
        with self._lock:
            if index not in self._packed:
                packed, flags = self.host_packed()
                self._packed[index] = (
                    torch.from_numpy(packed).to(device),
                    torch.from_numpy(flags).to(device),
                )
            return self._packed[index]

    def dense_fields(self, heads: int, *, dtype=torch.float32, device=None) -> torch.Tensor:
        """Materialise the equivalent one-hot ``(H, P, Np, Np)`` fields (for checks)."""
        table = torch.from_numpy(self.table.astype(np.int64))
        onehot = torch.zeros(self.n_slots + 1, self.patch_count, self.patch_count, dtype=dtype)
        index = torch.where(table == _lib.SLA_SLOT_NONE, torch.full_like(table, self.n_slots), table)
        onehot.scatter_(0, index.unsqueeze(0), 1.0)
        fields = onehot[: self.n_slots].unsqueeze(0).expand(heads, -1, -1, -1).contiguous()
        return fields if device is None else fields.to(device)


_status_words: dict[int, torch.Tensor] = {}
_status_lock = threading.Lock()


def _status_word(device: torch.device) -> torch.Tensor:
    index = torch.device(device).index
    with _status_lock:
        word = _status_words.get(index)
        if word is None:
            word = torch.zeros(1, dtype=torch.int32, device=device)
            _status_words[index] = word
        return word


def check_device_status(device=None) -> None:
    """Synchronise and raise if a bounded device wait gave up since the last check."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    word = _status_word(device)
    code = ctypes.c_int32()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        status = _lib.load().sla_read_status(ctypes.c_void_p(word.data_ptr()), ctypes.byref(code), ctypes.c_void_p(stream))
    if status != _lib.INTP_OK:
        raise RuntimeError(f"device wait failed: code {code.value:#x} ({_lib.status_string(status)})")


def _stride4(t: torch.Tensor):
    return _lib._Stride(*[int(s) for s in t.stride()])


class LookSlotFields:
    """Look fields ``(H, P, Np, Np)`` held per slot: ``fields[h, p, q, k] =
    values[h, p, slot(q, k)]``, zero where the pair has no slot.

    ``slots`` is the :class:`LookSlots` pair table, ``values`` a ``(H, P, S)``
    floating tensor with ``S = slots.n_slots`` (it may require grad).
    """

    def __init__(self, slots: LookSlots, values: torch.Tensor) -> None:
        if not isinstance(slots, LookSlots):
            raise ValueError("slots must be a LookSlots table")
        if not isinstance(values, torch.Tensor) or values.ndim != 3 or values.shape[-1] != slots.n_slots:
            raise ValueError("values must be a (H, P, n_slots) tensor")
        self.slots = slots
        self.values = values

    @property
    def shape(self) -> tuple[int, ...]:
        heads, poses, _ = self.values.shape
        return (heads, poses, self.slots.patch_count, self.slots.patch_count)

    def dense(self) -> torch.Tensor:
        """The equivalent ``(H, P, Np, Np)`` field tensor (for checks; Np^2 memory)."""
        table = torch.from_numpy(self.slots.table.astype(np.int64)).to(self.values.device)
        none = table == _lib.SLA_SLOT_NONE
        gathered = self.values[:, :, table.masked_fill(none, 0)]
        return gathered.masked_fill(none, 0.0)


def _validate(q, k, v, pose, fields, dense_bias):
    """The reference's checks, in its order (layers/triton_structured_look_attention.py:298-319)."""
    tensors = [q, k, v, pose] + ([fields] if isinstance(fields, torch.Tensor) else [])
    if isinstance(fields, LookSlotFields):
        tensors.append(fields.values)
    if dense_bias is not None:
        tensors.append(dense_bias)
    if not all(isinstance(t, torch.Tensor) and t.is_cuda for t in tensors):
        raise ValueError("structured Look attention requires CUDA tensors")
    if q.shape != k.shape or q.shape != v.shape or q.ndim != 4:
        raise ValueError("q, k, and v must share shape (B,H,N,D)")
    if pose.ndim != 4 or len(fields.shape) != 4:
        raise ValueError("pose and fields must have shapes (B,N,H,P) and (H,P,N,N)")
    batch, heads, sequence, head_dim = q.shape
    patch_count, poses = pose.shape[1], pose.shape[-1]
    if pose.shape != (batch, patch_count, heads, poses):
        raise ValueError("pose shape is inconsistent with q")
    if isinstance(fields, LookSlots):
        if fields.n_slots != poses or fields.patch_count != patch_count or fields.heads not in (None, heads):
            raise ValueError("fields shape is inconsistent with pose")
    elif isinstance(fields, LookSlotFields):
        if fields.shape != (heads, poses, patch_count, patch_count):
            raise ValueError("fields shape is inconsistent with pose")
        if fields.values.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ValueError("slot values must be float32, float16 or bfloat16")
    elif fields.shape != (heads, poses, patch_count, patch_count):
        raise ValueError("fields shape is inconsistent with pose")
    if dense_bias is not None and dense_bias.shape != (batch, heads, patch_count, patch_count):
        raise ValueError("dense_bias shape is inconsistent with q")
    if sequence != patch_count + 1:
        raise ValueError("sequence must be patch_count + one CLS token")
    if head_dim > 128:
        raise ValueError("head_dim above 128 is not supported")
    devices = {t.device for t in tensors}
    if len(devices) != 1:
        raise ValueError("all tensors must be on the same CUDA device")
    for t in (q, k, v):
        if t.dtype not in _DTYPE_CODE:
            raise ValueError("q, k, v must be float32, float16 or bfloat16")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k and v must share a dtype")


def _forward_args(q, k, v, pose, fields, scale, dense_bias, out, lse, kernel):
    """``sla_forward_args`` for these tensors; also returns the temporaries it points at."""
    batch, heads, sequence, head_dim = q.shape
    device = q.device
    args = _lib.SlaForwardArgs()
    args.batch, args.heads, args.seq, args.head_dim = batch, heads, sequence, head_dim
    args.scale = float(scale)
    args.dtype = _DTYPE_CODE[q.dtype]
    args.q, args.q_stride = q.data_ptr(), _stride4(q)
    args.k, args.k_stride = k.data_ptr(), _stride4(k)
    args.v, args.v_stride = v.data_ptr(), _stride4(v)
    args.out, args.out_stride = out.data_ptr(), _stride4(out)
    args.lse = lse.data_ptr() if lse is not None else None
    keep = []
    pose_f = pose if pose.dtype in _DTYPE_CODE else pose.float()
    keep.append(pose_f)
    args.poses = pose_f.shape[-1]
    args.pose, args.pose_stride, args.pose_dtype = pose_f.data_ptr(), _stride4(pose_f), _DTYPE_CODE[pose_f.dtype]
    if isinstance(fields, LookSlots):
        packed, flags = fields.device_packed(device)
        args.bias_mode = _lib.SLA_BIAS_SLOTS
        args.slots_packed, args.slot_tile_flags = packed.data_ptr(), flags.data_ptr()
    elif isinstance(fields, LookSlotFields):
        packed, flags = fields.slots.device_packed(device)
        values = fields.values
        args.bias_mode = _lib.SLA_BIAS_SLOT_FIELDS
        args.slots_packed, args.slot_tile_flags = packed.data_ptr(), flags.data_ptr()
        args.fields, args.fields_dtype = values.data_ptr(), _DTYPE_CODE[values.dtype]
        args.fields_stride = _lib._Stride(values.stride(0), values.stride(1), values.stride(2), 0)
        args.slots = fields.slots.n_slots
    else:
        fields_f = fields if fields.dtype in _DTYPE_CODE else fields.float()
        keep.append(fields_f)
        args.bias_mode = _lib.SLA_BIAS_FIELDS
        args.fields, args.fields_stride = fields_f.data_ptr(), _stride4(fields_f)
        args.fields_dtype = _DTYPE_CODE[fields_f.dtype]
    if dense_bias is not None:
        dense_f = dense_bias if dense_bias.dtype in _DTYPE_CODE else dense_bias.float()
        keep.append(dense_f)
        args.dense, args.dense_stride, args.dense_dtype = dense_f.data_ptr(), _stride4(dense_f), _DTYPE_CODE[dense_f.dtype]
    args.status = _status_word(device).data_ptr()
    if kernel not in _KERNELS:
        raise ValueError(f"kernel must be one of {sorted(_KERNELS)}")
    args.kernel = _KERNELS[kernel]
    return args, keep


def look_attention_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    pose: torch.Tensor,
    fields,
    *,
    scale: float,
    dense_bias: torch.Tensor | None = None,
    want_lse: bool = False,
    kernel: str = "auto",
    out: torch.Tensor | None = None,
):
    """Forward only.  Returns ``(out, lse_or_None)``.

    ``kernel`` selects the implementation: ``"auto"`` (tensor cores when the
    inputs qualify, else CUDA cores), ``"simt"`` or ``"tcgen05"`` (raises if
    the tensor-core path cannot take the inputs).
    """
    _validate(q, k, v, pose, fields, dense_bias)
    batch, heads, sequence, head_dim = q.shape
    device = q.device
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        raise ValueError("q, k, v need a unit stride on head_dim")
    if out is None:
        out = torch.empty((batch, heads, sequence, head_dim), dtype=q.dtype, device=device)
    elif out.shape != q.shape or out.dtype != q.dtype or out.device != device or out.stride(-1) != 1:
        raise ValueError("out must match q in shape, dtype and device with unit stride on head_dim")
    lse = torch.empty((batch, heads, sequence), dtype=torch.float32, device=device) if want_lse else None

    args, keep = _forward_args(q, k, v, pose, fields, scale, dense_bias, out, lse, kernel)
    lib = _lib.load()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        status = lib.sla_forward(ctypes.byref(args), ctypes.c_void_p(stream))
    _lib.check(status, "structured Look attention")
    return out, lse


def look_probability_score_grad(q, k, v, out, lse, grad_out, pose, slots: "LookSlots", *, scale):
    """The reference's probability / score-gradient pass
    (``_structured_look_probability_score_grad``,
    layers/triton_structured_look_attention.py:172-292) on the tensor cores:
    returns ``(probability, score_grad, grad_pose)`` with the first two
    ``(B, H, N, N)`` in q's dtype (views of row-padded buffers) and
    ``grad_pose`` ``(B, N-1, H, n_slots)`` float32, the per-slot sums of
    ``score_grad`` (the reference's pose gradient through one-hot fields).
    bf16 / f16, head_dim 64; anything else raises ValueError."""
    _validate(q, k, v, pose, slots, None)
    if not isinstance(slots, LookSlots):
        raise ValueError("look_probability_score_grad takes a LookSlots table")
    batch, heads, sequence, head_dim = q.shape
    device = q.device
    grad_out = grad_out.to(q.dtype)
    if grad_out.stride(-1) != 1:
        grad_out = grad_out.contiguous()
    ld = (sequence + 7) // 8 * 8
    probability = torch.empty(batch, heads, sequence, ld, dtype=q.dtype, device=device)
    score_grad = torch.empty_like(probability)
    dpose = torch.empty(batch, sequence - 1, heads, pose.shape[-1], dtype=torch.float32, device=device)
    fwd, keep = _forward_args(q, k, v, pose, slots, scale, None, out, lse, "auto")
    args = _lib.SlaProbabilityScoreGradArgs()
    args.fwd = fwd
    args.grad_out, args.grad_out_stride = grad_out.data_ptr(), _stride4(grad_out)
    args.probability, args.score_grad, args.ld = probability.data_ptr(), score_grad.data_ptr(), ld
    args.grad_pose = dpose.data_ptr()
    lib = _lib.load()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        status = lib.sla_probability_score_grad(ctypes.byref(args), ctypes.c_void_p(stream))
    del keep
    if status == _lib.INTP_ERR_UNSUPPORTED:
        raise ValueError("the probability / score-gradient pass takes bf16 / f16 inputs with head_dim 64")
    _lib.check(status, "structured Look attention probability / score gradient")
    return probability[..., :sequence], score_grad[..., :sequence], dpose


def look_attention_backward(q, k, v, out, lse, grad_out, pose, fields, *, scale, dense_bias=None,
                            needs=(True, True, True, True, True, True), kernel: str = "auto"):
    """Gradients of ``look_attention_forward`` (flash-style, from the forward's
    ``out`` and ``lse``).  Returns ``(dq, dk, dv, dpose, dfields, ddense)`` in the
    inputs' dtypes; entries whose ``needs`` flag is False, ``dfields`` for
    ``LookSlots`` fields (a table, not a tensor) and ``ddense`` without a dense
    bias are None.

    ``kernel``: ``"auto"`` takes the tensor-core backward (bf16 / f16,
    head_dim 64, slot tables, no dense bias) when it applies and the CUDA-core
    backward otherwise; ``"simt"`` forces the CUDA-core backward; ``"tcgen05"``
    raises when the tensor-core backward cannot take the inputs."""
    _validate(q, k, v, pose, fields, dense_bias)
    if kernel not in _KERNELS:
        raise ValueError(f"kernel must be one of {sorted(_KERNELS)}")
    device = q.device
    if grad_out.shape != q.shape or grad_out.device != device:
        raise ValueError("grad_output must match q in shape and device")
    if isinstance(fields, LookSlotFields):
        # Through the per-slot values pose . values (the SLOTS form), then the
        # chain rule back to pose and the slot values.
        sf = fields.values.float()
        per_slot = torch.einsum("bqhp,hps->bqhs", pose.float(), sf)
        want = needs[3] or needs[4]
        dq, dk, dv, dslot, _, ddense = look_attention_backward(
            q, k, v, out, lse, grad_out, per_slot, fields.slots, scale=scale, dense_bias=dense_bias,
            needs=(needs[0], needs[1], needs[2], want, False, needs[5]), kernel=kernel)
        dpose = torch.einsum("bqhs,hps->bqhp", dslot, sf).to(pose.dtype) if needs[3] else None
        dvalues = torch.einsum("bqhp,bqhs->hps", pose.float(), dslot).to(fields.values.dtype) if needs[4] else None
        return dq, dk, dv, dpose, dvalues, ddense
    grad_out = grad_out.to(q.dtype)
    if grad_out.stride(-1) != 1:
        grad_out = grad_out.contiguous()
    slots = isinstance(fields, LookSlots)
    batch, heads, sequence, head_dim = q.shape
    patches = sequence - 1
    f32 = dict(dtype=torch.float32, device=device)
    dq = torch.empty(q.shape, **f32) if needs[0] else None
    dk = torch.empty(q.shape, **f32) if needs[1] else None
    dv = torch.empty(q.shape, **f32) if needs[2] else None
    dpose = torch.empty(batch, patches, heads, pose.shape[-1], **f32) if needs[3] else None
    dfields = torch.zeros(fields.shape, **f32) if needs[4] and not slots else None
    ddense = torch.empty(batch, heads, patches, patches, **f32) if needs[5] and dense_bias is not None else None
    delta = torch.empty(batch, heads, sequence, **f32)
    pose_k = pose
    if slots and kernel != "simt" and (pose.dtype != torch.float32 or pose.stride(-1) != 1):
        pose_k = pose.float().contiguous()  # the tensor-core path copies fp32 pose rows
    fwd, keep = _forward_args(q, k, v, pose_k, fields, scale, dense_bias, out, lse, kernel)
    args = _lib.SlaBackwardArgs()
    args.fwd = fwd
    if slots and kernel != "simt":
        args.slots_packed_t = fields.device_packed_t(device).data_ptr()
    args.grad_out, args.grad_out_stride = grad_out.data_ptr(), _stride4(grad_out)
    for name, t in (("grad_q", dq), ("grad_k", dk), ("grad_v", dv), ("grad_pose", dpose), ("grad_fields", dfields),
                    ("grad_dense", ddense), ("delta", delta)):
        setattr(args, name, t.data_ptr() if t is not None else None)
    lib = _lib.load()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        status = lib.sla_backward(ctypes.byref(args), ctypes.c_void_p(stream))
    if status == _lib.INTP_ERR_UNSUPPORTED and kernel == "tcgen05":
        raise ValueError("the tensor-core backward takes bf16 / f16 inputs with head_dim 64, "
                         "a slot table and no dense bias")
    _lib.check(status, "structured Look attention backward")
    del keep
    return (dq.to(q.dtype) if dq is not None else None,
            dk.to(k.dtype) if dk is not None else None,
            dv.to(v.dtype) if dv is not None else None,
            dpose.to(pose.dtype) if dpose is not None else None,
            dfields.to(fields.dtype) if dfields is not None else None,
            ddense.to(dense_bias.dtype) if ddense is not None else None)


class _StructuredLookAttention(torch.autograd.Function):
    """Autograd wrapper (layers/triton_structured_look_attention.py:297-409): the
    forward keeps its LSE; the backward recomputes P from it on the GPU."""

    @staticmethod
    def forward(ctx, q, k, v, pose, fields_t, dense_bias, scale, slots):
        # fields_t: the dense fields (slots None), empty (LookSlots), or the
        # (H, P, S) slot values (LookSlotFields).
        fields = fields_t if slots is None else (slots if fields_t.numel() == 0 else LookSlotFields(slots, fields_t))
        dense = dense_bias if dense_bias.numel() else None
        out, lse = look_attention_forward(q, k, v, pose, fields, scale=scale, dense_bias=dense, want_lse=True)
        ctx.scale = scale
        ctx.slots = slots
        ctx.has_dense = dense is not None
        ctx.save_for_backward(q, k, v, pose, fields_t, dense_bias, out, lse)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, pose, fields_t, dense_bias, out, lse = ctx.saved_tensors
        slots = ctx.slots
        fields = fields_t if slots is None else (slots if fields_t.numel() == 0 else LookSlotFields(slots, fields_t))
        needs = ctx.needs_input_grad[:6]
        dq, dk, dv, dpose, dfields, ddense = look_attention_backward(
            q, k, v, out, lse, grad_output, pose, fields, scale=ctx.scale,
            dense_bias=dense_bias if ctx.has_dense else None, needs=needs)
        return dq, dk, dv, dpose, dfields, ddense, None, None


def structured_look_attention(q, k, v, pose, fields, *, scale, dense_bias=None):
    """Memory-bounded Look attention forward (layers/triton_structured_look_attention.py:412-424).

    A dense ``fields`` tensor that is a layer slice of a hooked Look layer's
    ``transformed_look_grids()`` result runs in its compact slot form
    (``look_registry``); any other dense tensor runs the general form."""
    from .look_registry import compact_fields

    fields = compact_fields(fields)
    values = fields.values if isinstance(fields, LookSlotFields) else fields
    if not torch.is_grad_enabled() or not any(
        t.requires_grad for t in (q, k, v, pose, values, dense_bias) if isinstance(t, torch.Tensor)
    ):
        out, _ = look_attention_forward(q, k, v, pose, fields, scale=scale, dense_bias=dense_bias)
        return out
    if dense_bias is None:
        dense_bias = q.new_empty(0)
    if isinstance(fields, LookSlotFields):
        return _StructuredLookAttention.apply(q, k, v, pose, fields.values, dense_bias, float(scale), fields.slots)
    if isinstance(fields, LookSlots):
        return _StructuredLookAttention.apply(q, k, v, pose, q.new_empty(0), dense_bias, float(scale), fields)
    return _StructuredLookAttention.apply(q, k, v, pose, fields, dense_bias, float(scale), None)
