"""Fast-path selection for dense Look fields, without editing the model.

The reference model builds its Look fields once per forward with
``SquarePatchDenseGridLook.transformed_look_grids()``
(layers/square_patch_dense_grid_look.py:357-379): an ``(H, S, T, Np, Np)``
tensor whose every ``(Np, Np)`` plane samples head ``h``'s Look grid at
per-pair geometry that depends only on the pair.  It flattens that tensor to
``(H, S*T, Np, Np)`` and hands each layer the slice ``fields[3l:3l+3]``
(model/deit_tiny_rot_hex_look.py:396-400) through
``block(..., structured_look=(pose, fields, dense))`` to
``structured_look_attention`` (layers/mini_vit.py:93-106).

Such a slice reaches the operator as a plain tensor.  This module recognises
it: ``install_look_bank_hook`` wraps the Look layer's
``transformed_look_grids`` so that each tensor it returns is registered,
keyed by its storage, together with the layer's pair geometry grouped into
slots (pairs whose sampling weights agree share a slot).  When
``structured_look_attention`` later receives a slice of a registered tensor
(same storage and version counter, the layer's ``(H, S*T, Np, Np)`` strides)
it runs the compact ``LookSlotFields(slots, values[h0:h0+H'])`` form, with
``values[h, p, s]`` gathered from the tensor itself at one representative pair
per slot, on the tensor-core kernel.  Anything not registered (or modified in
place since) stays on the general FIELDS path.

Slot grouping rounds the per-pair bilinear weights to 1e-4 (the same rule as
``share_vit.look_slot_basis``): pairs whose weights differ only by float32
noise in the angle fractions share a slot.  ``SlotGeometry.weight_error`` is
the largest L1 distance between a pair's weights and its slot
representative's over any plane, so every field value differs from the
reference's by at most ``weight_error * max|grid|``.
"""

from __future__ import annotations

import threading
import weakref
from dataclasses import dataclass, field

import numpy as np
import torch

from .look_attention import LookSlotFields, LookSlots

_TABLE_NAMES = ("look_radial0", "look_radial1", "look_angular0", "look_angular1", "look_radial_fraction",
                "look_angular_fraction", "look_valid")


@dataclass
class SlotGeometry:
    """A Look layer's pair geometry grouped into slots."""

    slots: LookSlots                 # (Np, Np) pair -> slot table
    representative: np.ndarray       # (S,) flat pair index q * Np + k of each slot's first pair
    planes: int                      # S*T field planes per head
    patches: int                     # Np
    weight_error: float              # max over pairs and planes of sum |w_pair - w_representative|
    _device_rep: dict = field(default_factory=dict)

    def representative_on(self, device: torch.device) -> torch.Tensor:
        key = (device.type, device.index)
        rep = self._device_rep.get(key)
        if rep is None:
            rep = torch.from_numpy(self.representative).to(device)
            self._device_rep[key] = rep
        return rep


def pair_weights_from_tables(tables: dict[str, torch.Tensor], radial_bins: int, direction_bins: int) -> np.ndarray:
    """Per-pair bilinear weights ``(Np*Np, planes, radial_bins*direction_bins)``
    (float64) of the sampling tables a Look layer registers
    (layers/square_patch_dense_grid_look.py:238-285): plane ``p`` of pair
    ``(q, k)`` reads cell ``r*A + a`` of the head's grid with the weight the
    four-tap formula of ``transformed_look_grids`` (:367-378) gives it."""
    r0, r1, a0, a1 = (tables[n].reshape(-1, *tables[n].shape[-2:]).long() for n in _TABLE_NAMES[:4])
    rw, aw = (tables[n].reshape(-1, *tables[n].shape[-2:]).double() for n in _TABLE_NAMES[4:6])
    valid = tables["look_valid"].reshape(-1, *tables["look_valid"].shape[-2:]).double()
    planes, n, _ = r0.shape
    cells = radial_bins * direction_bins
    dense = torch.zeros(planes, n, n, cells, dtype=torch.float64)
    for rr, ra, weight in ((r0, a0, (1 - rw) * (1 - aw)), (r0, a1, (1 - rw) * aw), (r1, a0, rw * (1 - aw)),
                           (r1, a1, rw * aw)):
        dense.scatter_add_(-1, (rr * direction_bins + ra).unsqueeze(-1), (weight * valid).unsqueeze(-1))
    return dense.permute(1, 2, 0, 3).reshape(n * n, planes, cells).numpy()


def group_pairs(weights: np.ndarray, *, decimals: int = 4, max_slots: int = 253) -> tuple[np.ndarray, np.ndarray, float]:
    """Groups pairs whose weights agree after rounding to ``decimals``.

    ``weights`` is ``(pairs, planes, cells)``.  Returns the flat slot table
    (uint8, 255 = the pair reads nothing), the first pair of every slot and
    the largest per-plane L1 distance between a pair and its slot's first pair."""
    pairs = weights.shape[0]
    flat = weights.reshape(pairs, -1)
    key = np.round(flat * 10.0 ** decimals).astype(np.int64)
    used = np.abs(key).sum(axis=1) > 0
    uniq, first_used, inverse = np.unique(key[used], axis=0, return_index=True, return_inverse=True)
    if uniq.shape[0] > max_slots:
        raise ValueError(f"Look geometry needs {uniq.shape[0]} slots, more than {max_slots}")
    # Slots numbered by their first pair, so the numbering follows the pair order.
    order = np.argsort(first_used)
    rank = np.empty_like(order)
    rank[order] = np.arange(order.size)
    used_rows = np.nonzero(used)[0]
    table = np.full(pairs, 255, dtype=np.uint8)
    table[used_rows] = rank[inverse.reshape(-1)].astype(np.uint8)
    representative = used_rows[first_used[order]].astype(np.int64)
    error = 0.0
    if used_rows.size:
        diff = np.abs(weights[used_rows] - weights[representative[table[used_rows]]])
        error = float(diff.sum(axis=-1).max())
    return table, representative, error


def slot_geometry_of(module) -> SlotGeometry:
    """Slot geometry of a ``SquarePatchDenseGridLook``-like layer from its
    registered sampling tables and grid shape (cached on the layer object)."""
    cached = getattr(module, "_intp_slot_geometry", None)
    if cached is not None:
        return cached
    grid = module.look_grid
    if grid.ndim != 3:
        raise ValueError("only (H, radial, direction) Look grids have a slot form")
    tables = {name: getattr(module, name).detach().cpu() for name in _TABLE_NAMES}
    weights = pair_weights_from_tables(tables, int(grid.shape[1]), int(grid.shape[2]))
    n = int(tables["look_valid"].shape[-1])
    table, representative, error = group_pairs(weights)
    n_slots = int(representative.size)
    geometry = SlotGeometry(LookSlots(table.reshape(n, n), max(n_slots, 1)), representative,
                            int(weights.shape[1]), n, error)
    object.__setattr__(module, "_intp_slot_geometry", geometry)
    return geometry


@dataclass
class _Entry:
    base: weakref.ref
    ptr: int
    version: int
    geometry: SlotGeometry
    values: torch.Tensor | None = None


class LookFieldRegistry:
    """Field tensors returned by hooked Look layers, keyed by storage pointer."""

    def __init__(self) -> None:
        self._entries: dict[int, _Entry] = {}
        self._lock = threading.Lock()
        self.hits = 0
        self.misses = 0

    def register(self, module, fields: torch.Tensor) -> None:
        """Record ``fields`` (the layer's ``transformed_look_grids()`` result)."""
        if not isinstance(fields, torch.Tensor) or not fields.is_cuda or not fields.is_contiguous():
            return
        if fields.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            return
        try:
            geometry = slot_geometry_of(module)
        except (AttributeError, ValueError):
            return
        heads = int(fields.shape[0])
        if fields.numel() != heads * geometry.planes * geometry.patches * geometry.patches:
            return
        ptr = fields.untyped_storage().data_ptr()
        with self._lock:
            for key in [k for k, e in self._entries.items() if e.base() is None]:
                del self._entries[key]
            self._entries[ptr] = _Entry(weakref.ref(fields), ptr, fields._version, geometry)

    def lookup(self, fields: torch.Tensor) -> LookSlotFields | None:
        """The compact form of ``fields`` when it is a layer slice of a
        registered, unmodified tensor; otherwise None."""
        if not isinstance(fields, torch.Tensor) or not fields.is_cuda or fields.ndim != 4:
            return None
        ptr = fields.untyped_storage().data_ptr()
        with self._lock:
            entry = self._entries.get(ptr)
        if entry is None:
            return None
        base = entry.base()
        if (base is None or base.untyped_storage().data_ptr() != ptr or fields._version != entry.version
                or base._version != entry.version or fields.dtype != base.dtype):
            self.misses += 1
            return None
        g = entry.geometry
        n, planes = g.patches, g.planes
        head_stride = planes * n * n
        offset = fields.storage_offset() - base.storage_offset()
        h = int(fields.shape[0])
        if (tuple(fields.shape[1:]) != (planes, n, n) or tuple(fields.stride()) != (head_stride, n * n, n, 1)
                or offset < 0 or offset % head_stride):
            self.misses += 1
            return None
        h0 = offset // head_stride
        if h0 + h > base.shape[0]:
            self.misses += 1
            return None
        if entry.values is None:
            flat = base.reshape(base.shape[0], planes, n * n)
            entry.values = flat.index_select(2, g.representative_on(base.device))
        self.hits += 1
        return LookSlotFields(g.slots, entry.values[h0:h0 + h])


REGISTRY = LookFieldRegistry()


def install_look_bank_hook(look_class) -> None:
    """Wraps ``look_class.transformed_look_grids`` (the reference's
    ``SquarePatchDenseGridLook``, layers/square_patch_dense_grid_look.py:357-379)
    so that every field tensor it returns is registered.  Idempotent; the
    wrapped method returns exactly what the original returns."""
    original = look_class.transformed_look_grids
    if getattr(original, "_intp_hooked", False):
        return

    def transformed_look_grids(self, *args, **kwargs):
        fields = original(self, *args, **kwargs)
        REGISTRY.register(self, fields)
        return fields

    transformed_look_grids._intp_hooked = True
    transformed_look_grids.__wrapped__ = original
    transformed_look_grids.__doc__ = original.__doc__
    look_class.transformed_look_grids = transformed_look_grids


def compact_fields(fields):
    """``fields`` in compact form when the registry knows it, else unchanged."""
    if isinstance(fields, torch.Tensor):
        compact = REGISTRY.lookup(fields)
        if compact is not None:
            return compact
    return fields
