"""Dense Look-grid sampling, host side: the oracle against the reference's own
outputs (tests/golden/dense_look_grid_reference.npz, made by make_golden.py
from layers/triton_dense_look_grid.py:19-49 and the tables of
layers/two_ring_circular_look.py:124-152), the product's table builder, the
wrapper's argument errors and the C ABI's checks (nothing is launched)."""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import _lib, look_sampling_tables
from intp_preliminary_b200.dense_look_grid import TABLE_NAMES, dense_look_grid_sample
from oracle.dense_look_grid import dense_look_grid_grad_np, dense_look_grid_np, sampling_tables_np

GOLDEN = np.load(Path(__file__).parent / "golden" / "dense_look_grid_reference.npz")


def _tables():
    return {name: GOLDEN[name] for name in TABLE_NAMES}


@pytest.mark.parametrize("tag", ["", "_bf16"])
def test_oracle_matches_reference_outputs(tag):
    grid = GOLDEN["grid"] if not tag else torch.from_numpy(GOLDEN["grid"]).to(torch.bfloat16).float().numpy()
    bias = dense_look_grid_np(grid, _tables())
    assert np.abs(bias - GOLDEN[f"bias{tag}"]).max() <= 2e-6
    grad = dense_look_grid_grad_np(GOLDEN["grad_out"], _tables())
    assert np.abs(grad - GOLDEN[f"grad_grid{tag}"]).max() <= 2e-5


@pytest.mark.parametrize("builder", ["product", "oracle"])
def test_table_builders_match_reference_tables(builder):
    coords = GOLDEN["coordinates"]
    tables = look_sampling_tables(torch.from_numpy(coords)) if builder == "product" else sampling_tables_np(coords)
    for name in TABLE_NAMES:
        got = np.asarray(tables[name])
        assert got.dtype == GOLDEN[name].dtype, name
        if name.endswith("fraction"):
            assert np.abs(got - GOLDEN[name]).max() <= 1e-6, name
        else:
            assert np.array_equal(got, GOLDEN[name]), name


def test_golden_case_exercises_every_corner():
    valid = GOLDEN["valid"]
    assert 0.3 < valid.mean() < 0.9
    assert set(np.unique(GOLDEN["radial0"][valid])) == {0, 1, 2, 3}
    assert (GOLDEN["radial1"][valid] == GOLDEN["radial0"][valid]).any()  # clamped at radius 4
    assert len(np.unique(GOLDEN["angular0"][valid])) == 12


def test_wrapper_errors_follow_the_reference():
    tables = [torch.from_numpy(GOLDEN[name]) for name in TABLE_NAMES]
    q = tables[0].shape[0]
    with pytest.raises(ValueError, match=r"dense Look grid must have shape \[B,Q,H,4,12\]"):
        dense_look_grid_sample(torch.zeros(1, q, 2, 4, 10), *tables)
    with pytest.raises(ValueError, match=r"Look sampling buffers must have shape \[Q,Q\]"):
        dense_look_grid_sample(torch.zeros(1, q + 1, 2, 4, 12), *tables)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        dense_look_grid_sample(torch.zeros(1, q, 2, 4, 12), *tables)


def _body(text, name):
    import re
    body = text[text.index(f"typedef struct {name}"):text.index(f"}} {name};")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    return re.findall(r"(\w+)(?:\[[^\]]*\])*\s*[;,]", body)


def test_dlg_struct_layout_matches_header():
    text = (Path(__file__).parent.parent / "include" / "intp_b200.h").read_text()
    assert _body(text, "dlg_args") == [f[0] for f in _lib.DlgArgs._fields_]
    assert _body(text, "dlg_grad_strides") == [f[0] for f in _lib.DlgGradStrides._fields_]


def test_dlg_host_side_argument_checks():
    lib = _lib.load()
    assert lib.dlg_forward(None, None) == _lib.INTP_ERR_ARGUMENT
    a = _lib.DlgArgs()
    a.batch, a.queries, a.heads, a.dtype = 0, 7, 3, _lib.INTP_F32
    assert lib.dlg_forward(ctypes.byref(a), None) == _lib.INTP_OK  # empty work, nothing launched
    a.batch, a.dtype = 2, 9
    assert lib.dlg_forward(ctypes.byref(a), None) == _lib.INTP_ERR_DTYPE
    a.dtype = _lib.INTP_BF16
    assert lib.dlg_forward(ctypes.byref(a), None) == _lib.INTP_ERR_ARGUMENT  # null tables
    fake = 1 << 20  # never dereferenced: each case below is rejected before a launch
    for name in TABLE_NAMES:
        setattr(a, name, fake)
    assert lib.dlg_forward(ctypes.byref(a), None) == _lib.INTP_ERR_ARGUMENT  # null grid / out
    strides = _lib.DlgGradStrides()
    assert lib.dlg_backward(ctypes.byref(a), None, ctypes.byref(strides), fake, None) == _lib.INTP_ERR_ARGUMENT
    a.queries = 1025
    assert lib.dlg_backward(ctypes.byref(a), fake, ctypes.byref(strides), fake, None) == _lib.INTP_ERR_UNSUPPORTED
