"""GPU parity of the negative-L1 kernel against the reference's golden outputs and
the float64 oracle (relative 1e-5, the bar for fp32 negative L1)."""

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import negative_l1_distance
from oracle.negative_l1 import negative_l1_np
from tests.golden_data import load

pytestmark = pytest.mark.gpu
NL1 = load("negative_l1_reference.npz")
RTOL = 1e-5


def _rel_err(actual: np.ndarray, expected: np.ndarray) -> float:
    scale = np.maximum(np.abs(expected), 1.0)
    return float((np.abs(actual - expected) / scale).max(initial=0.0))


@pytest.mark.parametrize("name", ["t7x11", "t37x67", "b432", "b1728"])
def test_golden(cuda_device, name):
    x = torch.from_numpy(NL1[f"{name}_x"]).to(cuda_device)
    w = torch.from_numpy(NL1[f"{name}_w"]).to(cuda_device)
    out = negative_l1_distance(x, w)
    assert out.dtype == torch.float32 and out.shape == (x.shape[0], w.shape[0])
    assert _rel_err(out.cpu().numpy(), NL1[f"{name}_out"]) <= RTOL
    assert _rel_err(out.cpu().numpy(), negative_l1_np(NL1[f"{name}_x"], NL1[f"{name}_w"])) <= RTOL


@pytest.mark.parametrize("rows,protos,features", [
    (1, 1, 1), (127, 63, 31), (129, 65, 33), (300, 576, 432), (257, 576, 1344), (64, 576, 1728), (5, 700, 336),
])
def test_ragged_shapes(cuda_device, rows, protos, features):
    g = torch.Generator().manual_seed(rows * 7 + protos)
    x = torch.randn(rows, features, generator=g)
    w = torch.randn(protos, features, generator=g) * 0.5
    out = negative_l1_distance(x.to(cuda_device), w.to(cuda_device)).cpu().numpy()
    assert _rel_err(out, negative_l1_np(x.numpy(), w.numpy())) <= RTOL


def test_empty_and_zero_features(cuda_device):
    x = torch.randn(0, 8, device=cuda_device)
    w = torch.randn(3, 8, device=cuda_device)
    assert negative_l1_distance(x, w).shape == (0, 3)
    out = negative_l1_distance(torch.randn(4, 0, device=cuda_device), torch.randn(3, 0, device=cuda_device))
    assert out.shape == (4, 3) and (out == 0).all()


def test_noncontiguous_and_half_inputs_are_converted(cuda_device):
    g = torch.Generator().manual_seed(2)
    x = torch.randn(40, 96, generator=g)
    w = torch.randn(50, 96, generator=g)
    out = negative_l1_distance(x.to(cuda_device).t().contiguous().t(), w.half().to(cuda_device))
    expected = negative_l1_np(x.numpy(), w.half().float().numpy())
    assert _rel_err(out.cpu().numpy(), expected) <= RTOL


def test_full_baseline_shape_properties(cuda_device):
    """The standalone projection at full size (M = 256*196, P = 576, F = 1728): sampled
    rows against the oracle, the identity d(w_p, w_p) = 0, and non-positivity."""
    g = torch.Generator(device=cuda_device).manual_seed(0)
    rows, protos, features = 256 * 196, 576, 1728
    x = torch.randn(rows, features, device=cuda_device, generator=g)
    w = torch.randn(protos, features, device=cuda_device, generator=g) * 0.5
    x[1000:1000 + protos] = w  # rows equal to the prototypes
    out = negative_l1_distance(x, w)
    assert (out <= 0).all()
    diag = out[1000:1000 + protos].diagonal()
    assert diag.abs().max().item() == 0.0
    sample = torch.tensor([0, 1, 777, 1500, 25000, rows - 1])
    expected = negative_l1_np(x[sample].cpu().numpy(), w.cpu().numpy())
    assert _rel_err(out[sample.to(cuda_device)].cpu().numpy(), expected) <= RTOL
