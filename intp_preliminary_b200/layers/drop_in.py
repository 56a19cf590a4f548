"""Put this package's operators under the reference's module names in a
running process, so that the reference's models run unchanged on them.

The reference imports its hot-path operators from three modules of its
``layers`` package: ``layers.triton_structured_look_attention``
(layers/mini_vit.py:94), ``layers.triton_negative_l1``
(layers/hex_rotating_harmonic_patch_embed.py:182) and
``layers.triton_dense_look_grid`` (layers/multiprobe_look.py:14,
layers/two_ring_circular_look.py:8).  ``install_drop_in()`` registers the
drop-in modules of ``intp_preliminary_b200.layers`` under those names in
``sys.modules`` and hooks the reference's ``SquarePatchDenseGridLook`` so
that the model's dense Look-field slices take the tensor-core path
(``look_registry``).  Call it before the reference's ``layers`` package is
imported; the reference's files stay as they are.

``polar_render="torch"`` also replaces ``layers.triton_polar_renderer`` (the
tokenizer's Triton renderer, outside this package's hot path) with the
reference's own PyTorch renderer, ``renderer(prototype)`` — what the
reference itself runs for CPU tensors (layers/triton_polar_renderer.py:160-164)
— so that no Triton kernel runs at all.
"""

from __future__ import annotations

import importlib
import sys
import types

from . import triton_dense_look_grid, triton_negative_l1, triton_structured_look_attention
from ..look_registry import install_look_bank_hook

_MODULES = {
    "layers.triton_structured_look_attention": triton_structured_look_attention,
    "layers.triton_negative_l1": triton_negative_l1,
    "layers.triton_dense_look_grid": triton_dense_look_grid,
}


def _torch_polar_renderer() -> types.ModuleType:
    module = types.ModuleType("layers.triton_polar_renderer")

    def triton_polar_render(prototype, renderer):
        """The reference's PyTorch polar renderer on any device."""
        return renderer(prototype)

    module.triton_polar_render = triton_polar_render
    module.__doc__ = "PyTorch polar renderer standing in for the reference's Triton one."
    return module


def install_drop_in(*, polar_render: str | None = "torch") -> dict[str, types.ModuleType]:
    """Registers the drop-in modules under the reference's names and hooks the
    Look bank.  Returns the ``sys.modules`` entries it set."""
    if polar_render not in (None, "torch"):
        raise ValueError("polar_render must be None or 'torch'")
    for name in _MODULES:
        current = sys.modules.get(name)
        if current is not None and current is not _MODULES[name]:
            raise RuntimeError(f"{name} is already imported; install the drop-in before the reference's layers")
    installed = dict(_MODULES)
    if polar_render == "torch":
        if "layers.triton_polar_renderer" in sys.modules and not getattr(
                sys.modules["layers.triton_polar_renderer"], "_intp_torch_renderer", False):
            raise RuntimeError("layers.triton_polar_renderer is already imported")
        renderer = sys.modules.get("layers.triton_polar_renderer") or _torch_polar_renderer()
        renderer._intp_torch_renderer = True
        installed["layers.triton_polar_renderer"] = renderer
    sys.modules.update(installed)
    look = importlib.import_module("layers.square_patch_dense_grid_look")
    install_look_bank_hook(look.SquarePatchDenseGridLook)
    package = sys.modules["layers"]
    for name, module in installed.items():
        setattr(package, name.rsplit(".", 1)[1], module)
    return installed
