"""GPU parity of dense Look-grid sampling (``dlg_forward`` / ``dlg_backward``)
against the reference's outputs (golden fixture) and the float64 oracle.

Tolerances: fp32 2e-6 max-abs on the bias (one rounding of a 4-term sum of
|grid| ~ 4 values) and 2e-5 on the gradient; bf16 / fp16 outputs within one
rounding of the float32 value (relative 2^-8 / 2^-11 plus 1e-6)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import dense_look_grid_backward, dense_look_grid_sample, hexgrid, look_sampling_tables
from intp_preliminary_b200.dense_look_grid import TABLE_NAMES
from intp_preliminary_b200.layers.triton_dense_look_grid import dense_look_grid_sample as drop_in
from oracle.dense_look_grid import dense_look_grid_grad_np, dense_look_grid_np

pytestmark = pytest.mark.gpu
GOLDEN = np.load(Path(__file__).parent / "golden" / "dense_look_grid_reference.npz")


def _golden_tables(device):
    return [torch.from_numpy(GOLDEN[name]).to(device) for name in TABLE_NAMES]


def _np_tables(tables):
    return {name: t.cpu().numpy() for name, t in zip(TABLE_NAMES, tables)}


def test_forward_and_grad_match_reference_fp32(cuda_device):
    tables = _golden_tables(cuda_device)
    grid = torch.from_numpy(GOLDEN["grid"]).to(cuda_device).requires_grad_(True)
    bias = drop_in(grid, *tables)
    assert bias.dtype == torch.float32 and bias.shape == GOLDEN["bias"].shape
    assert np.abs(bias.detach().cpu().numpy() - GOLDEN["bias"]).max() <= 2e-6
    bias.backward(torch.from_numpy(GOLDEN["grad_out"]).to(cuda_device))
    assert np.abs(grid.grad.cpu().numpy() - GOLDEN["grad_grid"]).max() <= 2e-5


@pytest.mark.parametrize("dtype,rel", [(torch.bfloat16, 2 ** -8), (torch.float16, 2 ** -11)])
def test_half_precision_grids(cuda_device, dtype, rel):
    tables = _golden_tables(cuda_device)
    grid = torch.from_numpy(GOLDEN["grid"]).to(cuda_device).to(dtype)
    bias = dense_look_grid_sample(grid, *tables)
    assert bias.dtype == dtype
    exact = dense_look_grid_np(grid.float().cpu().numpy(), _np_tables(tables))
    if dtype == torch.bfloat16:
        assert np.abs(exact - GOLDEN["bias_bf16"]).max() <= 2e-6  # same rounded grid as the reference case
    err = np.abs(bias.float().cpu().numpy() - exact)
    assert (err <= rel * np.abs(exact) + 1e-6).all(), err.max()


def test_strided_grid_tables_and_output(cuda_device):
    """A grid slice of a larger buffer (as multiprobe_look passes grids[:, :, :, s]
    before making it contiguous), tables that are slices of stacked buffers,
    and a transposed output view."""
    tables = _golden_tables(cuda_device)
    q = tables[0].shape[0]
    g = torch.Generator(cuda_device).manual_seed(3)
    big = torch.randn(3, q, 4, 2, 4, 12, device=cuda_device, generator=g)  # (B, Q, H, S, 4, 12)
    grid = big[:, :, :, 1]
    strided_tables = [torch.stack([torch.zeros_like(t), t], dim=-1)[..., 1] if i % 2 == 0
                      else t.t().contiguous().t() for i, t in enumerate(tables)]  # strides (2Q, 2) / (1, Q)
    assert not any(t.is_contiguous() for t in strided_tables)
    out = torch.empty(q, q, 3, 4, device=cuda_device).permute(2, 3, 0, 1)  # (B, H, Q, K) view
    from intp_preliminary_b200 import dense_look_grid_forward
    dense_look_grid_forward(grid, *strided_tables, out=out)
    exact = dense_look_grid_np(grid.cpu().numpy(), _np_tables(tables))
    assert np.abs(out.cpu().numpy() - exact).max() <= 2e-6


def test_layer_size_against_oracle_and_adjoint(cuda_device):
    """The half6d3r layer shape on the 14 x 14 lattice (B 64, H 3, Q 196):
    forward against the oracle, backward against the oracle on two images, and
    <forward(g), G> = <g, backward(G)> over the whole batch."""
    coords = torch.from_numpy(hexgrid.offset_row_lattice(14, 14)).float()
    tables = [t.to(cuda_device) for t in look_sampling_tables(coords).values()]
    nt = _np_tables(tables)
    g = torch.Generator(cuda_device).manual_seed(5)
    grid = torch.randn(64, 196, 3, 4, 12, device=cuda_device, generator=g)
    gout = torch.randn(64, 3, 196, 196, device=cuda_device, generator=g)
    bias = dense_look_grid_sample(grid, *tables)
    assert np.abs(bias.cpu().numpy() - dense_look_grid_np(grid.cpu().numpy(), nt)).max() <= 2e-6
    grad = dense_look_grid_backward(gout, *tables, grid_shape=grid.shape)
    exact = dense_look_grid_grad_np(gout[:2].cpu().numpy(), nt)
    assert np.abs(grad[:2].cpu().numpy() - exact).max() <= 2e-5
    lhs = (bias.double() * gout.double()).sum().item()
    rhs = (grid.double() * grad.double()).sum().item()
    assert abs(lhs - rhs) <= 1e-5 * max(1.0, abs(lhs))


def test_backward_is_deterministic(cuda_device):
    tables = _golden_tables(cuda_device)
    g = torch.Generator(cuda_device).manual_seed(7)
    gout = torch.randn(4, 3, tables[0].shape[0], tables[0].shape[0], device=cuda_device, generator=g)
    shape = (4, tables[0].shape[0], 3, 4, 12)
    a = dense_look_grid_backward(gout, *tables, grid_shape=shape)
    b = dense_look_grid_backward(gout, *tables, grid_shape=shape)
    assert torch.equal(a, b)


def test_rows_beyond_one_cta_and_empty_batch(cuda_device):
    """More (batch, head) rows than one forward / backward CTA takes (64 / 128),
    with a ragged last chunk; an empty batch launches nothing."""
    tables = _golden_tables(cuda_device)
    q = tables[0].shape[0]
    g = torch.Generator(cuda_device).manual_seed(9)
    grid = torch.randn(45, q, 3, 4, 12, device=cuda_device, generator=g)  # 135 rows
    gout = torch.randn(45, 3, q, q, device=cuda_device, generator=g)
    nt = _np_tables(tables)
    bias = dense_look_grid_sample(grid, *tables)
    assert np.abs(bias.cpu().numpy() - dense_look_grid_np(grid.cpu().numpy(), nt)).max() <= 2e-6
    grad = dense_look_grid_backward(gout, *tables, grid_shape=grid.shape)
    assert np.abs(grad.cpu().numpy() - dense_look_grid_grad_np(gout.cpu().numpy(), nt)).max() <= 2e-5
    empty = dense_look_grid_sample(grid[:0], *tables)
    assert empty.shape == (0, 3, q, q)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_contiguous_and_strided_bias_agree(cuda_device, dtype):
    """Q = 196 into a contiguous bias and into a view whose key stride is not 1:
    the arithmetic per element is the same, so the results are identical, and
    both agree with the oracle within one rounding."""
    from intp_preliminary_b200 import dense_look_grid_forward
    coords = torch.from_numpy(hexgrid.offset_row_lattice(14, 14)).float()
    tables = [t.to(cuda_device) for t in look_sampling_tables(coords).values()]
    g = torch.Generator(cuda_device).manual_seed(11)
    grid = torch.randn(5, 196, 3, 4, 12, device=cuda_device, generator=g).to(dtype)
    vec = dense_look_grid_forward(grid, *tables)
    strided = torch.empty(196, 5, 3, 196, dtype=dtype, device=cuda_device).permute(1, 2, 3, 0)  # key stride != 1
    dense_look_grid_forward(grid, *tables, out=strided)
    assert torch.equal(vec, strided)
    exact = dense_look_grid_np(grid.float().cpu().numpy(), _np_tables(tables))
    rel = {torch.float32: 1e-6, torch.bfloat16: 2 ** -8, torch.float16: 2 ** -11}[dtype]
    assert (np.abs(vec.float().cpu().numpy() - exact) <= rel * np.abs(exact) + 2e-6).all()
