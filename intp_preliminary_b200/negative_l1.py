"""Negative L1 distance projection on B200: the drop-in for
``layers/triton_negative_l1.py`` of the reference.

``negative_l1_distance(x, prototype)`` returns ``out[m, p] = -sum_f |x[m, f] -
prototype[p, f]|`` as a float32 ``(Q, P)`` tensor (layers/triton_negative_l1.py:233-241),
computed by the CUDA-core kernel of ``libintp_b200.so``.  Inputs are made
contiguous float32 first, as the reference wrapper does (:240).  There is no
CPU fallback: CPU tensors raise ``ValueError``.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib


def _validate(x: torch.Tensor, prototype: torch.Tensor) -> None:
    """The reference's checks (layers/triton_negative_l1.py:160-168)."""
    if x.ndim != 2 or prototype.ndim != 2:
        raise ValueError("expected x [Q,F] and prototype [H,F]")
    if x.shape[1] != prototype.shape[1]:
        raise ValueError("x and prototype feature dimensions differ")
    if not (x.is_cuda and prototype.is_cuda):
        raise ValueError("negative L1 distance requires CUDA tensors")
    if x.device != prototype.device:
        raise ValueError("x and prototype must be on the same CUDA device")


def negative_l1_forward(x: torch.Tensor, prototype: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """Forward only: ``-||x - w||_1`` for every row/prototype pair."""
    _validate(x, prototype)
    x = x.contiguous().float()
    prototype = prototype.contiguous().float()
    rows, features = x.shape
    protos = prototype.shape[0]
    if out is None:
        out = torch.empty((rows, protos), dtype=torch.float32, device=x.device)
    elif out.shape != (rows, protos) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32 (Q, P) tensor")
    lib = _lib.load()
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream(x.device).cuda_stream
        status = lib.nl1_forward(
            ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(prototype.data_ptr()), ctypes.c_void_p(out.data_ptr()),
            rows, protos, features, ctypes.c_void_p(stream),
        )
    _lib.check(status, "negative L1 distance")
    return out


def negative_l1_backward(x: torch.Tensor, prototype: torch.Tensor, grad_output: torch.Tensor,
                         needs=(True, True)):
    """``(grad_x, grad_prototype)`` of ``-||x - w||_1`` (layers/triton_negative_l1.py:55-154,
    189-230): with s = sign(x - w), sign(0) = 0, grad_x = -sum_p g s and
    grad_w = sum_m g s, float32."""
    _validate(x, prototype)
    x = x.contiguous().float()
    prototype = prototype.contiguous().float()
    grad_output = grad_output.contiguous().float()
    rows, features = x.shape
    protos = prototype.shape[0]
    if grad_output.shape != (rows, protos):
        raise ValueError("grad_output must be (Q, P)")
    gx = torch.empty_like(x) if needs[0] else None
    gw = torch.empty_like(prototype) if needs[1] else None
    if gx is None and gw is None:
        return None, None
    lib = _lib.load()
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream(x.device).cuda_stream
        status = lib.nl1_backward(
            ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(prototype.data_ptr()),
            ctypes.c_void_p(grad_output.data_ptr()), ctypes.c_void_p(gx.data_ptr() if gx is not None else None),
            ctypes.c_void_p(gw.data_ptr() if gw is not None else None), rows, protos, features,
            ctypes.c_void_p(stream))
    _lib.check(status, "negative L1 backward")
    return gx, gw


class _NegativeL1(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, prototype):
        ctx.save_for_backward(x, prototype)
        return negative_l1_forward(x, prototype)

    @staticmethod
    def backward(ctx, grad_output):
        x, prototype = ctx.saved_tensors
        gx, gw = negative_l1_backward(x, prototype, grad_output, needs=ctx.needs_input_grad[:2])
        return (gx.to(x.dtype) if gx is not None else None, gw.to(prototype.dtype) if gw is not None else None)


def negative_l1_distance(x: torch.Tensor, prototype: torch.Tensor) -> torch.Tensor:
    """Return ``-||x-w||_1`` as [Q,H] without a broadcast difference tensor."""
    if torch.is_grad_enabled() and (x.requires_grad or prototype.requires_grad):
        return _NegativeL1.apply(x, prototype)
    return negative_l1_forward(x, prototype)
