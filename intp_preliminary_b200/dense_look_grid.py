"""Dense Look-grid sampling on B200: the drop-in for ``layers/triton_dense_look_grid.py``
of the reference.

``dense_look_grid_sample(grid, radial0, radial1, angular0, angular1,
radial_fraction, angular_fraction, valid)`` bilinearly samples each query's
4 x 12 Look grid ``grid[b, q, h]`` at every key's (radius, angle) corners from
the (Q, Q) sampling tables and returns the dense attention bias (B, H, Q, Q) in
``grid.dtype`` (layers/triton_dense_look_grid.py:19-49 for the math, :114-150 /
:184-202 for the API).  The forward and the grid gradient run in
``libintp_b200.so`` (``dlg_forward`` / ``dlg_backward``); there is no CPU
fallback: CPU tensors raise ``ValueError``.

``look_sampling_tables(coordinates)`` builds the seven tables for a lattice the
way the reference's Look layers register them
(layers/two_ring_circular_look.py:124-152).
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_DTYPE_CODE = {torch.float32: _lib.INTP_F32, torch.float16: _lib.INTP_F16, torch.bfloat16: _lib.INTP_BF16}
_GRID_SHAPE_ERROR = "dense Look grid must have shape [B,Q,H,4,12]"
_TABLE_SHAPE_ERROR = "Look sampling buffers must have shape [Q,Q]"
TABLE_NAMES = ("radial0", "radial1", "angular0", "angular1", "radial_fraction", "angular_fraction", "valid")


def look_sampling_tables(coordinates: torch.Tensor) -> dict[str, torch.Tensor]:
    """Sampling tables of a lattice with unit spacing (host work, once per
    lattice): for the displacement of key k from query q, cells centred at radii
    1..4 (radial0 = floor(d - 1) clamped to 0..3, radial1 = radial0 + 1 clamped
    to 3, fraction d - 1 - floor(d - 1) clamped to [0, 1]) and 12 angular bins
    (angular0 = floor(12 angle / 2 pi) mod 12, angular1 = angular0 + 1 mod 12);
    valid where 0 < d <= 4.  Restates layers/two_ring_circular_look.py:124-152."""
    xy = torch.as_tensor(coordinates, dtype=torch.float32).cpu()
    if xy.ndim != 2 or xy.shape[1] != 2:
        raise ValueError("coordinates must be (Q, 2)")
    rel = xy.unsqueeze(0) - xy.unsqueeze(1)
    distance = rel.norm(dim=-1)
    angle = torch.remainder(torch.atan2(rel[..., 1], rel[..., 0]), 2.0 * math.pi)
    radial = distance - 1.0
    radial0 = radial.floor().clamp(0, 3).long()
    angular = angle / (2.0 * math.pi) * 12.0
    angular0 = angular.floor().long() % 12
    return {
        "radial0": radial0,
        "radial1": (radial0 + 1).clamp_max(3),
        "angular0": angular0,
        "angular1": (angular0 + 1) % 12,
        "radial_fraction": (radial - radial.floor()).clamp(0.0, 1.0),
        "angular_fraction": angular - angular.floor(),
        "valid": (distance > 0) & (distance <= 4.0),
    }


def _prepare(grid: torch.Tensor, tables) -> tuple[list[torch.Tensor], int]:
    """The reference's checks (layers/triton_dense_look_grid.py:127-132), then
    the table dtypes the kernel reads (int64 indices, float32 fractions, one
    byte per valid flag)."""
    if grid.ndim != 5 or tuple(grid.shape[-2:]) != (4, 12):
        raise ValueError(_GRID_SHAPE_ERROR)
    queries = grid.shape[1]
    if any(tuple(t.shape) != (queries, queries) for t in tables):
        raise ValueError(_TABLE_SHAPE_ERROR)
    if not grid.is_cuda or any(not t.is_cuda for t in tables):
        raise ValueError("dense Look grid sampling requires CUDA tensors")
    if any(t.device != grid.device for t in tables):
        raise ValueError("grid and sampling buffers must be on the same CUDA device")
    if grid.dtype not in _DTYPE_CODE:
        raise ValueError("dense Look grid must be float32, float16 or bfloat16")
    r0, r1, a0, a1, rw, aw, valid = tables
    prepared = [t if t.dtype == torch.int64 else t.long() for t in (r0, r1, a0, a1)]
    prepared += [t if t.dtype == torch.float32 else t.float() for t in (rw, aw)]
    prepared.append(valid.view(torch.uint8) if valid.dtype == torch.bool else (valid != 0).view(torch.uint8))
    return prepared, queries


def _args(grid: torch.Tensor, tables: list[torch.Tensor], out: torch.Tensor | None) -> _lib.DlgArgs:
    a = _lib.DlgArgs()
    a.batch, a.queries, a.heads = grid.shape[0], grid.shape[1], grid.shape[2]
    a.dtype = _DTYPE_CODE[grid.dtype]
    a.grid = grid.data_ptr()
    for i, s in enumerate(grid.stride()):
        a.grid_stride[i] = s
    for name, t in zip(TABLE_NAMES, tables):
        setattr(a, name, t.data_ptr())
    for i, t in enumerate(tables):
        a.table_stride[i][0], a.table_stride[i][1] = t.stride()
    if out is not None:
        a.out = out.data_ptr()
        for i, s in enumerate(out.stride()):
            a.out_stride[i] = s
    return a


def dense_look_grid_forward(grid: torch.Tensor, radial0: torch.Tensor, radial1: torch.Tensor,
                            angular0: torch.Tensor, angular1: torch.Tensor, radial_fraction: torch.Tensor,
                            angular_fraction: torch.Tensor, valid: torch.Tensor, *,
                            out: torch.Tensor | None = None) -> torch.Tensor:
    """Forward only: the (B, H, Q, Q) bias in ``grid.dtype`` (any grid and table
    strides; ``out`` may be a strided (B, H, Q, Q) view)."""
    tables, queries = _prepare(grid, (radial0, radial1, angular0, angular1, radial_fraction, angular_fraction, valid))
    batch, heads = grid.shape[0], grid.shape[2]
    if out is None:
        out = torch.empty(batch, heads, queries, queries, dtype=grid.dtype, device=grid.device)
    elif tuple(out.shape) != (batch, heads, queries, queries) or out.dtype != grid.dtype or out.device != grid.device:
        raise ValueError("out must be a (B, H, Q, Q) tensor of the grid's dtype and device")
    args = _args(grid, tables, out)
    with torch.cuda.device(grid.device):
        status = _lib.load().dlg_forward(ctypes.byref(args),
                                         ctypes.c_void_p(torch.cuda.current_stream(grid.device).cuda_stream))
    _lib.check(status, "dense Look grid sampling")
    return out


def dense_look_grid_backward(grad_out: torch.Tensor, radial0: torch.Tensor, radial1: torch.Tensor,
                             angular0: torch.Tensor, angular1: torch.Tensor, radial_fraction: torch.Tensor,
                             angular_fraction: torch.Tensor, valid: torch.Tensor, *,
                             grid_shape, dtype: torch.dtype | None = None) -> torch.Tensor:
    """Gradient with respect to the grid, (B, Q, H, 4, 12) contiguous: each cell
    sums grad_out[b, h, q, k] times the corner weights of the keys that sample it
    (layers/triton_dense_look_grid.py:152-181), in float32 and a fixed order."""
    dtype = dtype or grad_out.dtype
    if grad_out.dtype != dtype:
        grad_out = grad_out.to(dtype)
    batch, queries, heads = grid_shape[0], grid_shape[1], grid_shape[2]
    shape_probe = torch.empty(batch, queries, heads, 4, 12, dtype=dtype, device=grad_out.device)
    tables, _ = _prepare(shape_probe, (radial0, radial1, angular0, angular1, radial_fraction, angular_fraction,
                                       valid))
    if tuple(grad_out.shape) != (batch, heads, queries, queries):
        raise ValueError("grad_output must be (B, H, Q, Q)")
    grad_grid = shape_probe
    args = _args(grad_grid, tables, None)
    strides = _lib.DlgGradStrides()
    for i, s in enumerate(grad_out.stride()):
        strides.stride[i] = s
    with torch.cuda.device(grad_out.device):
        status = _lib.load().dlg_backward(
            ctypes.byref(args), ctypes.c_void_p(grad_out.data_ptr()), ctypes.byref(strides),
            ctypes.c_void_p(grad_grid.data_ptr()),
            ctypes.c_void_p(torch.cuda.current_stream(grad_out.device).cuda_stream))
    _lib.check(status, "dense Look grid backward")
    return grad_grid


class _DenseLookGridSample(torch.autograd.Function):
    """Autograd as the reference's ``_DenseLookGridSample`` (:114-181): a
    gradient for the grid only."""

    @staticmethod
    def forward(ctx, grid, radial0, radial1, angular0, angular1, radial_fraction, angular_fraction, valid):
        out = dense_look_grid_forward(grid, radial0, radial1, angular0, angular1, radial_fraction,
                                      angular_fraction, valid)
        ctx.grid_shape = tuple(grid.shape)
        ctx.grid_dtype = grid.dtype
        ctx.save_for_backward(radial0, radial1, angular0, angular1, radial_fraction, angular_fraction, valid)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        grad_grid = dense_look_grid_backward(grad_output, *ctx.saved_tensors, grid_shape=ctx.grid_shape,
                                             dtype=ctx.grid_dtype)
        return (grad_grid,) + (None,) * 7


def dense_look_grid_sample(grid: torch.Tensor, radial0: torch.Tensor, radial1: torch.Tensor,
                           angular0: torch.Tensor, angular1: torch.Tensor, radial_fraction: torch.Tensor,
                           angular_fraction: torch.Tensor, valid: torch.Tensor) -> torch.Tensor:
    """Public API of the reference (layers/triton_dense_look_grid.py:184-202):
    grid [B,Q,H,4,12] -> bias [B,H,Q,Q] in grid.dtype, differentiable in grid."""
    return _DenseLookGridSample.apply(grid, radial0, radial1, angular0, angular1, radial_fraction,
                                      angular_fraction, valid)
