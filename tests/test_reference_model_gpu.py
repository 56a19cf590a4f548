"""The reference's own models, unchanged, on this package's operators.

The reference's ``layers``/``model``/``utils`` packages are imported from
baseline/_ref (installed by ``sh baseline/install_reference.sh <checkout>``;
git-ignored, it travels with the working tree).  ``install_drop_in()`` puts
this package's operators under the reference's module names
(``layers.triton_structured_look_attention``, ``layers.triton_negative_l1``,
``layers.triton_dense_look_grid``), hooks the reference's Look bank, and
replaces the reference's Triton polar renderer by its own PyTorch renderer.
Nothing in the reference's files changes.

* ``DeiTTinyRotHexLook`` half6d3r (model/deit_tiny_rot_hex_look.py:19-488):
  fp32 logits against the reference's CPU logits (golden fixture) at 1e-4;
  every layer's dense field slice is recognised (registry hits) and, under
  bf16 autocast, runs on the tensor-core kernel (profiler kernel names), with
  the per-layer attention outputs within 2e-2 of the float64 oracle on the
  layer's own inputs.
* ``HexViTClassifier`` (model/hex_vit_classifier.py:171-249) runs unchanged on
  the GPU with the drop-ins installed and matches its CPU run.
* ``HexRotatingHarmonicPatchEmbed`` with ``match_metric="relative_l1"``
  (layers/hex_rotating_harmonic_patch_embed.py:166-195) reaches
  ``negative_l1_distance`` through the drop-in module and matches its CPU path.
* ``sample_pose_grids`` (layers/multiprobe_look.py:37-53) reaches
  ``dense_look_grid_sample`` through the drop-in module and matches the oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from intp_preliminary_b200 import check_device_status
from intp_preliminary_b200.look_registry import REGISTRY
from intp_preliminary_b200.share_vit import ShareViTHalf6d3r
from tests.golden_data import load

ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "baseline" / "_ref"
GOLD = load("share_vit_reference.npz")
HALF6D3R = dict(use_pos_embed=True, directions=6, global_directions=12, angular_bins_per_radius=3,
                look_compact_variable_rings=True, tokenizer_null_initial_score=0.0)

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not (REF / "model" / "deit_tiny_rot_hex_look.py").exists(),
                       reason="reference not installed in baseline/_ref (sh baseline/install_reference.sh <checkout>)"),
]


def _reference_names(name: str) -> bool:
    return name.split(".")[0] in ("layers", "model", "utils")


@pytest.fixture(scope="module")
def ref():
    """The reference's modules imported from baseline/_ref with the drop-ins installed."""
    saved_modules = {k: v for k, v in sys.modules.items() if _reference_names(k)}
    for key in saved_modules:
        del sys.modules[key]
    sys.path.insert(0, str(REF))
    try:
        from intp_preliminary_b200.layers.drop_in import install_drop_in

        install_drop_in(polar_render="torch")
        import layers.hex_rotating_harmonic_patch_embed as harmonic
        import layers.mini_vit as mini_vit
        import layers.multiprobe_look as multiprobe
        import model.deit_tiny_rot_hex_look as deit
        import model.hex_vit_classifier as hexvit

        yield dict(deit=deit, hexvit=hexvit, harmonic=harmonic, multiprobe=multiprobe, mini_vit=mini_vit)
    finally:
        sys.path.remove(str(REF))
        for key in [k for k in sys.modules if _reference_names(k)]:
            del sys.modules[key]
        sys.modules.update(saved_modules)


def _half6d3r(ref, device):
    """The reference model with the weights of the golden fixture's seeded init."""
    weights = ShareViTHalf6d3r(precision="fp32").init_weights(seed=int(GOLD["weight_seed"]),
                                                               look_grid_std=float(GOLD["look_grid_std"]))
    model = ref["deit"].DeiTTinyRotHexLook(**HALF6D3R).eval()
    model.load_state_dict(weights.state_dict(), strict=True)
    return model.to(device)


def _images(device, count=2, seed=None):
    g = torch.Generator().manual_seed(int(GOLD["image_seed"]) if seed is None else seed)
    return torch.randn(count, 3, 224, 224, generator=g).to(device)


def test_half6d3r_fp32_logits_match_reference(ref, cuda_device):
    model = _half6d3r(ref, cuda_device)
    hits = REGISTRY.hits
    with torch.no_grad():
        logits = model(_images(cuda_device)).cpu().numpy()
    check_device_status(cuda_device)
    assert REGISTRY.hits - hits == 12, "every layer's field slice should take the compact path"
    np.testing.assert_allclose(logits, GOLD["logits"], atol=1e-4, rtol=1e-4)


def test_half6d3r_bf16_runs_on_the_tensor_core_kernel(ref, cuda_device, monkeypatch):
    from oracle.look_attention import look_attention_np

    model = _half6d3r(ref, cuda_device)
    shim = sys.modules["layers.triton_structured_look_attention"]
    original = shim.structured_look_attention
    captured = []

    def capture(q, k, v, pose, fields, *, scale, dense_bias=None):
        out = original(q, k, v, pose, fields, scale=scale, dense_bias=dense_bias)
        if len(captured) in (0, 11):
            captured.append(tuple(t.detach().float().cpu() for t in (q, k, v, pose, fields, out)) + (scale,))
        else:
            captured.append(None)
        return out

    monkeypatch.setattr(shim, "structured_look_attention", capture)
    images = _images(cuda_device, count=4, seed=23)
    hits = REGISTRY.hits
    from torch.profiler import ProfilerActivity, profile

    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            logits = model(images)
            torch.cuda.synchronize(cuda_device)
    check_device_status(cuda_device)
    assert REGISTRY.hits - hits == 12
    assert torch.isfinite(logits).all()
    names = [e.name for e in prof.events()]
    if names:  # the profiler saw the GPU: the attention ran on a tensor-core kernel only
        tensor_core = sum("sla_tc_kernel" in n or "sla_short_kernel" in n for n in names)
        assert tensor_core == 12, sorted(set(names))
        assert not any("sla_simt_kernel" in n for n in names)
    for item in (captured[0], captured[11]):
        q, k, v, pose, fields, out, scale = item
        for b in range(q.shape[0]):
            exact = look_attention_np(q[b:b + 1].numpy(), k[b:b + 1].numpy(), v[b:b + 1].numpy(),
                                      pose[b:b + 1].numpy(), fields.numpy(), scale=scale)
            err = float(np.abs(out[b:b + 1].numpy() - exact).max())
            assert err <= 2e-2, err


def test_hex_vit_classifier_runs_unchanged(ref, cuda_device):
    torch.manual_seed(3)
    model = ref["hexvit"].HexViTClassifier(img_size=32, num_classes=10, position_mode="learned+look").eval()
    images = torch.randn(2, 3, 32, 32, generator=torch.Generator().manual_seed(4))
    with torch.no_grad():
        expected = model(images)
        got = model.to(cuda_device)(images.to(cuda_device)).cpu()
    torch.testing.assert_close(got, expected, atol=1e-4, rtol=1e-4)


def test_harmonic_l1_tokenizer_reaches_the_drop_in(ref, cuda_device):
    embed = ref["harmonic"].HexRotatingHarmonicPatchEmbed(
        img_size=224, in_chans=3, embed_dim=192, lattice_stride=18, kernel_sizes=(24, 12), bases=96,
        directions=6, global_directions=12, angular_bins_per_radius=3, prototype_chunk_size=16,
        null_initial_score=0.0, pose_softmax=True, use_null=True, match_metric="relative_l1").eval()
    torch.manual_seed(5)
    with torch.no_grad():
        embed.prototype.normal_(0, 0.5)
    images = torch.randn(2, 3, 224, 224, generator=torch.Generator().manual_seed(6))
    with torch.no_grad():
        expected = embed(images)
        got = embed.to(cuda_device)(images.to(cuda_device)).cpu()
    scale = expected.abs().max().item()
    assert (got - expected).abs().max().item() <= 1e-4 * max(scale, 1.0)


def test_sample_pose_grids_reaches_the_drop_in(ref, cuda_device):
    from oracle.dense_look_grid import dense_look_grid_np

    model = ref["deit"].DeiTTinyRotHexLook(**HALF6D3R).eval()
    look = model.look_bank.to(cuda_device)
    n = look.num_patches
    g = torch.Generator().manual_seed(8)
    grids = torch.randn(2, n, 3, 2, 4, 12, generator=g)
    got = ref["multiprobe"].sample_pose_grids(grids.to(cuda_device), look, image=True).cpu().numpy()
    names = ("look_radial0", "look_radial1", "look_angular0", "look_angular1", "look_radial_fraction",
             "look_angular_fraction", "look_valid")
    expected = 0.0
    for scale in range(2):
        tables = {name.removeprefix("look_"): getattr(look, name)[scale, 0].cpu().numpy() for name in names}
        expected = expected + dense_look_grid_np(grids[:, :, :, scale].numpy(), tables)
    assert np.abs(got - expected).max() <= 2e-5
