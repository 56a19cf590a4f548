"""SHARE-ViT half6d3r DeiT-Tiny inference on the B200 Look-attention kernels.

This is the caller side of the hot path: the full forward of the reference's
``DeiTTinyRotHexLook`` in its half6d3r configuration (model/deit_tiny_rot_hex_look.py:19-488
with ``use_pos_embed=True, directions=6, global_directions=12,
angular_bins_per_radius=3, look_compact_variable_rings=True``), for inference.
Parameter and persistent-buffer names and shapes equal the reference's, so a
reference ``state_dict`` loads with ``strict=True``.

Forward, per batch of images (B, 3, 224, 224):

1. Hex patch gather (reflect padding + circular supports of 24 and 12 px on
   the 195-centre staggered lattice, layers/hex_patch_geometry.py:82-90),
   cover-weighted and flattened (layers/rotating_dot_product.py:9-13).  The
   tokenizer and the Look bank sample the same supports with the same cover
   (layers/square_patch_dense_grid_look.py:287-314), so one gather serves both.
2. One GEMM per support against the polar-rendered prototypes of both the
   tokenizer (96 bases x 6 directions) and the Look bank (36 heads x 6
   directions); the rendered prototypes depend only on the weights and are
   cached (layers/hex_rotating_polar_patch_embed.py:111-124 render).
3. Tokenizer: pose softmax with a learned null over the 6 directions, then
   cos/sin harmonic moments -> 192-d tokens (layers/hex_rotating_harmonic_patch_embed.py:153-242).
4. Look bank: null softmax over the 12 (scale, direction) responses per head
   -> pose (B, 195, 36, 12) (layers/square_patch_dense_grid_look.py:339-355).
5. Look fields in SLOTS form: the reference's fields (36, 12, 195, 195)
   (:357-379) are bilinear samples of each head's 4x12 grid at pair geometry
   that depends only on the pair; pairs with identical sampling weights share
   a slot, so the per-query Look value per slot is pose @ F_slots and the
   attention kernel reads it through a (195, 195) uint8 slot table.  In
   bf16 mode the attention takes pose and F_slots themselves
   (``LookSlotFields``) and forms pose @ F_slots per query tile in shared
   memory; the (B, 195, 36, S) per-slot values are never written.
6. 12 pre-norm transformer blocks (layers/mini_vit.py:138-170) whose attention
   is ``look_attention_forward`` (the tensor-core kernel for bf16), final
   LayerNorm and the classifier on the CLS token.

``precision="bf16"`` runs the GEMMs and the attention in bf16 (fp32 softmaxes,
LayerNorms and residual stream, like the reference under bf16 autocast) and is
the benchmark mode; ``precision="fp32"`` runs everything in fp32 (attention on
the CUDA-core kernel) and is the parity mode.
"""

from __future__ import annotations

import math
import threading
from typing import NamedTuple

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from .look_attention import LookSlotFields, LookSlots, look_attention_forward
from .share_vit_ops import (GatherPlan, add_layernorm, embed_post, gather_patches, gather_plan, linear_bias,
                            linear_gelu, linear_residual_layernorm, tokenizer_gemm)

IMAGE_SIZE = 224
IN_CHANS = 3
EMBED_DIM = 192
DEPTH = 12
HEADS = 3
KERNEL_SIZES = (24, 12)
LATTICE_STRIDE = 18
BASES = 96
DIRECTIONS = 6
GLOBAL_DIRECTIONS = 12
RADIAL_BINS = 12
ANGULAR_BINS_PER_RADIUS = 3
LOOK_HEADS = DEPTH * HEADS
LOOK_RADIAL = 2 * len(KERNEL_SIZES)          # 4
LOOK_DIRECTION_BINS = GLOBAL_DIRECTIONS      # 12
LOOK_SCALES = (1.0, 0.5)
LOOK_RADIUS = 4.0


# ----------------------------------------------------------------------------- geometry tables
def _disk_offsets(kernel: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Pixel (column, row) indices of a kernel x kernel square inside its
    inscribed circle, row-major (utils/hex_idx_genr.py:5-19)."""
    col = torch.arange(kernel).repeat(kernel, 1)       # col[i, j] = j
    centred = col.float() - (kernel - 1) / 2
    radius = torch.sqrt(centred * centred + centred.T * centred.T)
    inside = radius < kernel / 2
    return col[inside], col.T[inside]


def _lattice_starts(stride: int) -> tuple[torch.Tensor, torch.Tensor, int, int, int, int]:
    """Top-left sample offsets of the staggered hex lattice (utils/hex_idx_genr.py:21-55)."""
    step_x = stride // 2
    step_y = round(stride * (3 ** 0.5 / 2))
    n_x = math.ceil(IMAGE_SIZE / step_x) + 1
    n_y = math.ceil(IMAGE_SIZE / step_y) + 1
    xs, ys = _staggered(n_x, n_y, step_x, step_y, torch.int64)
    return xs, ys, n_x, n_y, step_x, step_y


def _staggered(n_x: int, n_y: int, step_x, step_y, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """Column-zig-zag lattice: pairs of rows, odd columns shifted by step_y;
    an odd final row keeps every other column."""
    row_x = torch.arange(n_x, dtype=dtype) * step_x
    row_y = torch.zeros(n_x, dtype=dtype)
    row_y[1::2] += step_y
    pairs = n_y // 2
    xs = row_x.repeat(pairs, 1)
    ys = row_y.repeat(pairs, 1) + torch.arange(pairs, dtype=dtype).unsqueeze(-1) * (2 * step_y)
    xs, ys = xs.reshape(-1), ys.reshape(-1)
    if n_y % 2:
        extra_x = xs[:n_x:2]
        xs = torch.cat((xs, extra_x))
        ys = torch.cat((ys, torch.zeros_like(extra_x) + (n_y - 1) * step_y))
    return xs, ys


class LookPose(NamedTuple):
    """Look inputs of the attention layers in SLOT_FIELDS form: ``pose`` (B, N,
    36, P) after the Look bank's null softmax and ``fields`` (36, P, S), the
    value of every slot for each head and pose."""

    pose: torch.Tensor
    fields: torch.Tensor


class HexSupport:
    """Gather tables of one circular support size (layers/hex_patch_geometry.py:10-90)."""

    def __init__(self, kernel: int):
        self.kernel = kernel
        cols, rows = _disk_offsets(kernel)
        xs, ys, n_x, n_y, step_x, step_y = _lattice_starts(LATTICE_STRIDE)
        self.pad_x = ((n_x - 1) * step_x + kernel - IMAGE_SIZE + 1) // 2
        self.pad_y = ((n_y - 1) * step_y + kernel - IMAGE_SIZE + 1) // 2
        self.sample_x = xs[:, None] + cols[None, :]   # rows of the padded image
        self.sample_y = ys[:, None] + rows[None, :]   # columns of the padded image
        centre = (kernel - 1) / 2.0
        self.centres_xy = torch.stack(
            (ys.float() - self.pad_y + centre, xs.float() - self.pad_x + centre), dim=-1)
        # offsets of the samples from the support centre: (row - c, col - c)
        self.offsets_xy = torch.stack((rows.float() - centre, cols.float() - centre), dim=-1)
        cx, cy = _staggered(n_x, n_y, 0.5, 3 ** 0.5 * 0.5, torch.float32)
        self.unit_xy = torch.stack((cx, cy), dim=-1)  # unit lattice coordinates of the centres

    @property
    def samples(self) -> int:
        return int(self.sample_x.shape[1])


class PolarTables:
    """Bilinear (radius, rotated angle) sampling of a compact polar prototype on
    one support (layers/hex_rotating_polar_patch_embed.py:11-124, forward only)."""

    def __init__(self, support: HexSupport):
        counts = torch.tensor([ANGULAR_BINS_PER_RADIUS * (r + 1) for r in range(RADIAL_BINS)], dtype=torch.long)
        offsets = torch.cat((torch.zeros(1, dtype=torch.long), counts.cumsum(0)))
        self.stored = int(offsets[-1])  # 234
        x, y = support.offsets_xy[:, 0], support.offsets_xy[:, 1]
        radius = torch.sqrt(x.square() + y.square())
        turn = torch.remainder(torch.atan2(y, x), 2 * math.pi) / (2 * math.pi)
        radial = (radius * RADIAL_BINS / (support.kernel / 2) - 0.5).clamp(0, RADIAL_BINS - 1)
        r0 = radial.floor().long()
        r1 = (r0 + 1).clamp_max(RADIAL_BINS - 1)
        shifts = (torch.arange(DIRECTIONS) * (2 * math.pi / GLOBAL_DIRECTIONS))[:, None] / (2 * math.pi)

        def angular(ring):
            count = counts[ring]
            position = torch.remainder(turn[None] - shifts, 1.0) * count[None]
            raw = position.floor()
            a0 = torch.remainder(raw.long(), count[None])
            a1 = torch.remainder(a0 + 1, count[None])
            return offsets[ring][None] + a0, offsets[ring][None] + a1, position - raw

        self.i00, self.i01, self.f0 = angular(r0)
        self.i10, self.i11, self.f1 = angular(r1)
        self.fr = radial - r0
        self.cover = torch.cos(radius * math.pi / support.kernel).clamp_min(0)

    def render(self, prototype: torch.Tensor) -> torch.Tensor:
        """(P, C, stored) compact prototypes -> (P, D, C, M) rendered supports."""
        p00, p01 = prototype[..., self.i00], prototype[..., self.i01]
        p10, p11 = prototype[..., self.i10], prototype[..., self.i11]
        f0, f1 = self.f0[None, None], self.f1[None, None]
        low = p00 * (1 - f0) + p01 * f0
        high = p10 * (1 - f1) + p11 * f1
        fr = self.fr[None, None, None]
        return (low * (1 - fr) + high * fr).permute(0, 2, 1, 3)


def look_sampling_tables(unit_xy: torch.Tensor):
    """Per pair (query, key), scale and source direction: the 4 bilinear taps
    into a head's 4 x 12 Look grid and their weights, zero outside the scale's
    radius (layers/square_patch_dense_grid_look.py:238-285, float32 like the
    reference so bin edges resolve identically).  Returns index (S*T, Np, Np, 4)
    into the flattened grid and weight (S*T, Np, Np, 4)."""
    relative = unit_xy.unsqueeze(0) - unit_xy.unsqueeze(1)
    distance = relative.norm(dim=-1)
    angle = torch.remainder(torch.atan2(relative[..., 1], relative[..., 0]), 2.0 * math.pi)
    step = 2.0 * math.pi / GLOBAL_DIRECTIONS
    index, weight = [], []
    for scale in LOOK_SCALES:
        radius = LOOK_RADIUS * scale
        position = distance / radius * LOOK_RADIAL - 1.0
        r0 = position.floor().clamp(0, LOOK_RADIAL - 1).long()
        r1 = (r0 + 1).clamp_max(LOOK_RADIAL - 1)
        rw = (position - position.floor()).clamp(0.0, 1.0)
        valid = ((distance > 0) & (distance <= radius)).float()
        for direction in range(DIRECTIONS):
            rel = torch.remainder(angle - direction * step, 2.0 * math.pi)
            apos = rel / (2.0 * math.pi) * LOOK_DIRECTION_BINS
            a0 = apos.floor().long() % LOOK_DIRECTION_BINS
            a1 = (a0 + 1) % LOOK_DIRECTION_BINS
            aw = apos - apos.floor()
            index.append(torch.stack((r0 * LOOK_DIRECTION_BINS + a0, r0 * LOOK_DIRECTION_BINS + a1,
                                      r1 * LOOK_DIRECTION_BINS + a0, r1 * LOOK_DIRECTION_BINS + a1), dim=-1))
            weight.append(torch.stack(((1.0 - rw) * (1.0 - aw), (1.0 - rw) * aw, rw * (1.0 - aw), rw * aw), dim=-1)
                          * valid.unsqueeze(-1))
    return torch.stack(index), torch.stack(weight)


def look_slot_basis(unit_xy: torch.Tensor, max_slots: int = 93):
    """Compress the Look fields' pair geometry into slots.

    fields[h, p, q, k] = sum_g B[p, q, k, g] * grid[h, g] with B the bilinear
    sampling weights of ``look_sampling_tables``.  Pairs whose 12 x 48 weight
    matrices agree to 1e-4 share a slot (float32 noise in the bilinear angle
    fractions otherwise splits identical geometry; merged pairs' fields differ
    by at most 1e-4 of a grid value); all-zero pairs get no slot.
    Returns (slot table (Np, Np) uint8 with 255 = none, basis (P=12, G=48, S)).
    """
    index, weight = look_sampling_tables(unit_xy)
    st, n, _, _ = index.shape
    dense = torch.zeros(st, n, n, LOOK_RADIAL * LOOK_DIRECTION_BINS, dtype=torch.float64)
    dense.scatter_add_(-1, index, weight.double())
    per_pair = dense.permute(1, 2, 0, 3).reshape(n * n, st * LOOK_RADIAL * LOOK_DIRECTION_BINS)
    key = torch.round(per_pair * 1e4).to(torch.int64)
    nonzero = key.abs().sum(dim=1) > 0
    uniq, inverse = torch.unique(key[nonzero], dim=0, return_inverse=True)
    if uniq.shape[0] > max_slots:
        raise ValueError(f"Look geometry needs {uniq.shape[0]} slots, more than {max_slots}")
    table = torch.full((n * n,), 255, dtype=torch.uint8)
    table[nonzero] = inverse.to(torch.uint8)
    # basis per slot: first pair of each class (classes agree to 1e-4)
    first = torch.full((uniq.shape[0],), -1, dtype=torch.long)
    rows = torch.nonzero(nonzero).squeeze(1)
    first.scatter_reduce_(0, inverse, rows, reduce="amin", include_self=False)
    basis = per_pair[first].reshape(-1, st, LOOK_RADIAL * LOOK_DIRECTION_BINS)  # (S, P, G)
    return table.reshape(n, n).numpy(), basis.permute(1, 2, 0).float().contiguous()  # (P, G, S)


def _reflect(index: torch.Tensor, size: int) -> torch.Tensor:
    """Source index of a reflect-padded coordinate (edge not repeated, like F.pad mode="reflect")."""
    index = index.abs()
    return torch.where(index >= size, 2 * (size - 1) - index, index)


# ----------------------------------------------------------------------------- modules
class _RotatingHarmonicTokenizer(nn.Module):
    """Parameters of layers/hex_rotating_harmonic_patch_embed.py (prototype, null, bias)."""

    def __init__(self):
        super().__init__()
        self.prototype = nn.Parameter(torch.zeros(BASES, IN_CHANS, 234))
        self.null_score = nn.Parameter(torch.zeros(BASES))
        self.output_bias = nn.Parameter(torch.zeros(EMBED_DIM))


class _LookBank(nn.Module):
    """Parameters and persistent buffers of layers/square_patch_dense_grid_look.py."""

    def __init__(self, centres_xy: torch.Tensor, unit_xy: torch.Tensor):
        super().__init__()
        self.match_prototype = nn.Parameter(torch.zeros(LOOK_HEADS, IN_CHANS, 234))
        self.null_score = nn.Parameter(torch.zeros(LOOK_HEADS))
        self.look_grid = nn.Parameter(torch.zeros(LOOK_HEADS, LOOK_RADIAL, LOOK_DIRECTION_BINS))
        self.register_buffer("patch_centers_xy", centres_xy.clone(), persistent=True)
        self.register_buffer("patch_coordinates_xy", unit_xy.clone(), persistent=True)


class _Attention(nn.Module):
    def __init__(self):
        super().__init__()
        self.qkv = nn.Linear(EMBED_DIM, 3 * EMBED_DIM)
        self.proj = nn.Linear(EMBED_DIM, EMBED_DIM)


class _Mlp(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(EMBED_DIM, 4 * EMBED_DIM)
        self.fc2 = nn.Linear(4 * EMBED_DIM, EMBED_DIM)


class _Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.norm1 = nn.LayerNorm(EMBED_DIM, eps=1e-6)
        self.attn = _Attention()
        self.norm2 = nn.LayerNorm(EMBED_DIM, eps=1e-6)
        self.mlp = _Mlp()


class ShareViTHalf6d3r(nn.Module):
    """Inference-only SHARE-ViT half6d3r DeiT-Tiny with B200 Look attention."""

    def __init__(self, num_classes: int = 100, *, precision: str = "bf16"):
        super().__init__()
        if precision not in ("bf16", "fp32"):
            raise ValueError("precision must be 'bf16' or 'fp32'")
        self.precision = precision
        self.supports = [HexSupport(k) for k in KERNEL_SIZES]
        self.polar = [PolarTables(s) for s in self.supports]
        n_patches = int(self.supports[0].sample_x.shape[0])
        self.num_patches = n_patches
        self.patch_embed = _RotatingHarmonicTokenizer()
        self.cls_token = nn.Parameter(torch.zeros(1, 1, EMBED_DIM))
        self.pos_embed = nn.Parameter(torch.zeros(1, n_patches + 1, EMBED_DIM))
        self.blocks = nn.ModuleList(_Block() for _ in range(DEPTH))
        self.norm = nn.LayerNorm(EMBED_DIM, eps=1e-6)
        self.head = nn.Linear(EMBED_DIM, num_classes)
        self.look_bank = _LookBank(self.supports[0].centres_xy, self.supports[0].unit_xy)
        slots, basis = look_slot_basis(self.supports[0].unit_xy)
        self.look_slots = LookSlots(slots, basis.shape[-1], heads=HEADS)
        self.register_buffer("look_basis", basis, persistent=False)            # (12, 48, S)
        reference_mass = self.polar[0].cover.sum()
        for i, polar in enumerate(self.polar):
            self.register_buffer(f"cover_{i}", polar.cover * (reference_mass / polar.cover.sum()), persistent=False)
            self.register_buffer(f"sample_x_{i}", self.supports[i].sample_x, persistent=False)
            self.register_buffer(f"sample_y_{i}", self.supports[i].sample_y, persistent=False)
        # Fused gather: per patch and feature (support blocks of channel-major
        # samples, the order of `_patches`), the pixel offset inside one image
        # after reflect padding, and the cover weight.
        index_parts, weight_parts = [], []
        for i, support in enumerate(self.supports):
            rows = _reflect(support.sample_x - support.pad_x, IMAGE_SIZE)
            cols = _reflect(support.sample_y - support.pad_y, IMAGE_SIZE)
            pixel = rows * IMAGE_SIZE + cols
            for c in range(IN_CHANS):
                index_parts.append(pixel + c * IMAGE_SIZE * IMAGE_SIZE)
                weight_parts.append(getattr(self, f"cover_{i}"))
        self.register_buffer("pixel_index", torch.cat(index_parts, dim=1).to(torch.int32).contiguous(), persistent=False)
        self.register_buffer("pixel_weight", torch.cat(weight_parts).float().contiguous(), persistent=False)
        # Shared-memory plan of the same gather: groups of 6 consecutive patches
        # (part of a column strip of the hex lattice, at most 1740 16-byte units:
        # 27.2 KB of shared memory, 8 CTAs per SM).
        plan = gather_plan(self.pixel_index, group_patches=6)
        self.register_buffer("gather_stage_offset", plan.stage_offset, persistent=False)
        self.register_buffer("gather_stage_begin", plan.stage_begin, persistent=False)
        self.register_buffer("gather_local_index", plan.local_index, persistent=False)
        self._gather_plan_sizes = (plan.group_patches, plan.max_stage, plan.max_offset)
        theta = torch.arange(DIRECTIONS) * (2 * math.pi / GLOBAL_DIRECTIONS)
        self.register_buffer("direction_coefficients", torch.stack((torch.cos(theta), torch.sin(theta)), -1),
                             persistent=False)
        self._cache_lock = threading.Lock()
        self._cache: dict = {}
        # When set to a list, forward() appends (start, stop) CUDA events around
        # every attention launch (used by the benchmark to time the kernel in place).
        self.attention_events: list | None = None
        # When set to a list, the bf16 forward appends each layer's attention
        # arguments (q, k, v as views of a copy of that layer's qkv buffer, pose,
        # fields, scale) so that the launches can be replayed on their own.
        self.attention_inputs: list | None = None

    # ------------------------------------------------------------------ weights
    def init_weights(self, seed: int = 0, look_grid_std: float = 0.02) -> "ShareViTHalf6d3r":
        """Deterministic random init with the reference's distributions
        (layers/mini_vit.py:173-184, model/deit_tiny_rot_hex_look.py:157-160,
        prototypes ~ N(0, 0.02)), plus a non-zero Look grid ~ N(0, look_grid_std)
        so the Look bias is active.  Drawn on the CPU from one generator."""
        g = torch.Generator().manual_seed(seed)

        def tn(shape, std=0.02):
            t = torch.empty(shape)
            nn.init.trunc_normal_(t, std=std, generator=g)
            return t

        with torch.no_grad():
            for name, param in self.named_parameters():
                if name.endswith("bias") or name.endswith("null_score"):
                    val = torch.zeros(param.shape)
                elif ".norm" in name or name.startswith("norm."):
                    val = torch.ones(param.shape)
                elif name in ("patch_embed.prototype", "look_bank.match_prototype"):
                    val = torch.randn(param.shape, generator=g) * 0.02
                elif name == "look_bank.look_grid":
                    val = torch.randn(param.shape, generator=g) * look_grid_std
                else:
                    val = tn(param.shape)
                param.copy_(val.to(param.device))
        self.invalidate_cache()
        return self

    def invalidate_cache(self) -> None:
        with self._cache_lock:
            self._cache.clear()

    def _weights_key(self):
        return tuple((p.data_ptr(), p._version) for p in (self.patch_embed.prototype, self.look_bank.match_prototype,
                                                          self.look_bank.look_grid))

    def _rendered(self, device, dtype):
        """Per support: (792, F) matrix [tokenizer 96x6 ; Look bank 36x6] of
        rendered prototypes (cached per weight version)."""
        key = ("rendered", device, dtype, self._weights_key())
        with self._cache_lock:
            hit = self._cache.get(key)
        if hit is not None:
            return hit
        mats = []
        for polar in self.polar:
            parts = []
            for proto in (self.patch_embed.prototype, self.look_bank.match_prototype):
                rendered = polar.render(proto.detach().float().cpu())          # (P, D, C, M)
                parts.append(rendered.reshape(-1, rendered.shape[2] * rendered.shape[3]))
            mats.append(torch.cat(parts).to(device=device, dtype=dtype).contiguous())
        with self._cache_lock:
            self._cache = {k: v for k, v in self._cache.items() if k[0] != "rendered"}
            self._cache[key] = mats
        return mats

    # ------------------------------------------------------------------ forward
    def _patches(self, image: torch.Tensor, index: int) -> torch.Tensor:
        support = self.supports[index]
        padded = F.pad(image, (support.pad_y, support.pad_y, support.pad_x, support.pad_x), mode="reflect")
        gathered = padded[..., getattr(self, f"sample_x_{index}"), getattr(self, f"sample_y_{index}")]
        weighted = gathered.transpose(1, 2) * getattr(self, f"cover_{index}")     # (B, N, C, M)
        return weighted.flatten(2)

    @torch.no_grad()
    def embed(self, image: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Tokens (B, N, 192) and Look pose weights (B, N, 36, 12), both fp32."""
        if image.ndim != 4 or tuple(image.shape[1:]) != (IN_CHANS, IMAGE_SIZE, IMAGE_SIZE):
            raise ValueError(f"expected images (B, {IN_CHANS}, {IMAGE_SIZE}, {IMAGE_SIZE})")
        cdt = torch.bfloat16 if self.precision == "bf16" else torch.float32
        batch, n = image.shape[0], self.num_patches
        image = image.float()
        mats = self._rendered(image.device, cdt)
        score = None
        look_resp = []
        for s in range(len(self.supports)):
            patch = self._patches(image, s).to(cdt).reshape(batch * n, -1)
            resp = (patch @ mats[s].T).float()                                     # (B*N, 792)
            tok = resp[:, : BASES * DIRECTIONS]
            score = tok if score is None else score + tok
            look_resp.append(resp[:, BASES * DIRECTIONS:].reshape(batch, n, LOOK_HEADS, DIRECTIONS))
        # tokenizer: null softmax over directions, cos/sin moments
        score = score.reshape(batch, n, BASES, DIRECTIONS)
        null = self.patch_embed.null_score.float()[None, None, :, None].expand(batch, n, BASES, 1)
        weights = torch.cat((score, null), -1).softmax(-1)[..., :-1]
        tokens = torch.einsum("bnpd,dc->bnpc", weights, self.direction_coefficients).reshape(batch, n, EMBED_DIM)
        tokens = tokens + self.patch_embed.output_bias
        # Look bank pose: (B, N, 36, 2 scales x 6 directions) with a null route per head
        look = torch.stack(look_resp, dim=3).reshape(batch, n, LOOK_HEADS, 2 * DIRECTIONS)
        lnull = self.look_bank.null_score.float()[None, None, :, None].expand(batch, n, LOOK_HEADS, 1)
        pose = torch.cat((look, lnull), -1).softmax(-1)[..., :-1]                 # (B, N, 36, 12)
        return tokens, pose

    def _fused_embed_weights(self, device, dtype=torch.bfloat16):
        """(W, F): the (576 + 2*216, F0 + F1) bf16 matrix of one GEMM that gives the
        tokenizer scores summed over both supports and the Look-bank responses of
        each support, and the per-slot Look fields (36, 12, S) fp32 (cached per
        weight version)."""
        key = ("fused", device, dtype, self._weights_key())
        with self._cache_lock:
            hit = self._cache.get(key)
        if hit is not None:
            return hit
        mats = self._rendered(device, dtype)
        tok, look = BASES * DIRECTIONS, LOOK_HEADS * DIRECTIONS
        f0, f1 = mats[0].shape[1], mats[1].shape[1]
        w = torch.zeros(tok + 2 * look, f0 + f1, dtype=dtype, device=device)
        w[:tok, :f0], w[:tok, f0:] = mats[0][:tok], mats[1][:tok]
        w[tok:tok + look, :f0] = mats[0][tok:]
        w[tok + look:, f0:] = mats[1][tok:]
        fields = self.slot_fields().to(device=device, dtype=torch.float32).contiguous()
        hit = (w, fields)
        with self._cache_lock:
            self._cache = {k: v for k, v in self._cache.items() if k[0] != "fused"}
            self._cache[key] = hit
        return hit

    def _tokenizer_weights(self, device):
        """The fused GEMM's weight with the Look rows ordered head by head: row
        576 + 12 h + 6 s + d holds support s's direction-d response of Look head h
        (in ``_fused_embed_weights`` it is row 576 + 216 s + 6 h + d), so one
        head's 12 poses are 12 consecutive accumulator columns."""
        w, fields = self._fused_embed_weights(device)
        key = ("tokenizer", device, self._weights_key())
        with self._cache_lock:
            hit = self._cache.get(key)
        if hit is not None:
            return hit, fields
        tok = BASES * DIRECTIONS
        h = torch.arange(LOOK_HEADS).view(-1, 1, 1)
        s_ = torch.arange(2).view(1, -1, 1)
        d = torch.arange(DIRECTIONS).view(1, 1, -1)
        look_rows = (tok + s_ * LOOK_HEADS * DIRECTIONS + h * DIRECTIONS + d).reshape(-1)
        order = torch.cat((torch.arange(tok), look_rows)).to(device)
        hit = w.index_select(0, order).contiguous()
        with self._cache_lock:
            self._cache = {k: v for k, v in self._cache.items() if k[0] != "tokenizer"}
            self._cache[key] = hit
        return hit, fields

    @torch.no_grad()
    def embed_fused(self, image: torch.Tensor, *, per_slot_values: bool = False, fused_tokenizer: bool = True):
        """bf16 tokenizer + Look bank on the fused kernels: the residual stream
        x (B, N+1, 192) fp32 with CLS and position embedding, and the Look
        inputs of the 12 attention layers.  Default: a ``LookPose`` - the Look
        pose (B, N, 36, 12) after the null softmax plus the (36, 12, S) slot
        values; each attention forms its per-slot values itself
        (``LookSlotFields``).  ``per_slot_values=True``: the per-slot Look values
        (B, N, 36, S) fp32 - a view of a (B, 36, N, S) buffer, so each head's
        rows are contiguous.  Same math as ``embed`` + ``look_values``."""
        if image.ndim != 4 or tuple(image.shape[1:]) != (IN_CHANS, IMAGE_SIZE, IMAGE_SIZE):
            raise ValueError(f"expected images (B, {IN_CHANS}, {IMAGE_SIZE}, {IMAGE_SIZE})")
        batch, n = image.shape[0], self.num_patches
        image = image.float().contiguous()
        w, fields = self._fused_embed_weights(image.device)
        plan = GatherPlan(self.gather_stage_offset, self.gather_stage_begin, self.gather_local_index,
                          *self._gather_plan_sizes)
        patches = gather_patches(image, self.pixel_index, self.pixel_weight, plan=plan)
        x = torch.empty(batch, n + 1, EMBED_DIM, dtype=torch.float32, device=image.device)
        if fused_tokenizer and not per_slot_values:
            # one tcgen05 kernel: the GEMM and the softmaxes from its fp32 accumulators
            wt, _ = self._tokenizer_weights(image.device)
            look_pose = torch.empty(batch, n, LOOK_HEADS, 2 * DIRECTIONS, dtype=torch.float32, device=image.device)
            tokenizer_gemm(patches, wt, batch=batch, patches_per_image=n, bases=BASES, directions=DIRECTIONS,
                           look_heads=LOOK_HEADS, look_poses=2 * DIRECTIONS,
                           token_null=self.patch_embed.null_score.detach().float().contiguous(),
                           direction_coef=self.direction_coefficients.contiguous(),
                           output_bias=self.patch_embed.output_bias.detach().float().contiguous(),
                           cls=self.cls_token.detach().float().reshape(-1).contiguous(),
                           pos_embed=self.pos_embed.detach().float().reshape(n + 1, EMBED_DIM).contiguous(),
                           look_null=self.look_bank.null_score.detach().float().contiguous(), x=x,
                           look_pose=look_pose)
            return x, LookPose(look_pose, fields)
        resp = patches @ w.t()
        values = look_pose = None
        if per_slot_values:
            values = torch.empty(batch, LOOK_HEADS, n, fields.shape[-1], dtype=torch.float32, device=image.device)
        else:
            look_pose = torch.empty(batch, n, LOOK_HEADS, 2 * DIRECTIONS, dtype=torch.float32, device=image.device)
        embed_post(resp, batch=batch, patches=n, bases=BASES, directions=DIRECTIONS, look_heads=LOOK_HEADS,
                   look_poses=2 * DIRECTIONS, token_null=self.patch_embed.null_score.detach().float().contiguous(),
                   direction_coef=self.direction_coefficients.contiguous(),
                   output_bias=self.patch_embed.output_bias.detach().float().contiguous(),
                   cls=self.cls_token.detach().float().reshape(-1).contiguous(),
                   pos_embed=self.pos_embed.detach().float().reshape(n + 1, EMBED_DIM).contiguous(),
                   look_null=self.look_bank.null_score.detach().float().contiguous(), slot_fields=fields,
                   x=x, values=values, look_pose=look_pose)
        if per_slot_values:
            return x, values.permute(0, 2, 1, 3)
        return x, LookPose(look_pose, fields)

    def _layer_look(self, look, layer: int):
        """(pose, fields) argument pair of attention layer ``layer`` for Look
        inputs from ``embed_fused``: SLOT_FIELDS form for a ``LookPose``, SLOTS
        form for per-slot values."""
        heads = slice(HEADS * layer, HEADS * (layer + 1))
        if isinstance(look, LookPose):
            return look.pose[:, :, heads], LookSlotFields(self.look_slots, look.fields[heads])
        return look[:, :, heads], self.look_slots

    @torch.no_grad()
    def trunk_fused(self, x: torch.Tensor, values, *, cls_only: bool = False,
                    linears: str = "tcgen05") -> torch.Tensor:
        """The 12 blocks and the final LayerNorm in bf16 on the fused kernels.
        ``linears="tcgen05"``: proj and fc2 are tcgen05 GEMMs whose epilogue adds
        the residual and applies the next LayerNorm, fc1 one whose epilogue applies
        GELU, qkv one with only the bias.  ``linears="cublas"``: cuBLAS linears with
        separate add + LayerNorm and GELU passes.  Look attention writes
        token-major output.  ``values`` is the Look input from ``embed_fused``.
        ``x`` is updated in place.  Returns the normalised tokens (B, N+1, 192)
        bf16, or only the CLS rows (B, 192) when ``cls_only``."""
        if linears not in ("tcgen05", "cublas"):
            raise ValueError("linears must be 'tcgen05' or 'cublas'")
        if linears == "tcgen05":
            return self._trunk_tcgen05(x, values, cls_only=cls_only)
        batch, n1 = x.shape[0], x.shape[1]
        rows = batch * n1
        head_dim = EMBED_DIM // HEADS
        weights = self._trunk_weights(torch.bfloat16)
        scale = 1.0 / math.sqrt(head_dim)
        events = self.attention_events
        attn = torch.empty(batch, n1, HEADS, head_dim, dtype=torch.bfloat16, device=x.device)
        attn_bhnd = attn.permute(0, 2, 1, 3)
        y = None
        for layer, blk in enumerate(self.blocks):
            w_qkv, b_qkv, w_proj, b_proj, w_fc1, b_fc1, w_fc2, b_fc2 = weights[layer]
            h = add_layernorm(x, y, blk.norm1.weight, blk.norm1.bias, 1e-6)
            qkv = F.linear(h, w_qkv, b_qkv).view(batch, n1, 3, HEADS, head_dim)
            q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
            pose_l, fields_l = self._layer_look(values, layer)
            if events is not None:
                start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
            look_attention_forward(q, k, v, pose_l, fields_l, scale=scale, out=attn_bhnd)
            if events is not None:
                stop.record()
                events.append((start, stop))
            y = F.linear(attn.view(rows, EMBED_DIM), w_proj, b_proj)
            h = add_layernorm(x, y, blk.norm2.weight, blk.norm2.bias, 1e-6)
            y = F.linear(F.gelu(F.linear(h, w_fc1, b_fc1)), w_fc2, b_fc2)
        if cls_only:
            return add_layernorm(x[:, 0], y.view(batch, n1, EMBED_DIM)[:, 0], self.norm.weight, self.norm.bias, 1e-6)
        return add_layernorm(x, y, self.norm.weight, self.norm.bias, 1e-6).view(batch, n1, EMBED_DIM)

    def _trunk_tcgen05(self, x: torch.Tensor, values, *, cls_only: bool) -> torch.Tensor:
        batch, n1 = x.shape[0], x.shape[1]
        rows = batch * n1
        head_dim = EMBED_DIM // HEADS
        weights = self._trunk_weights(torch.bfloat16)
        scale = 1.0 / math.sqrt(head_dim)
        events = self.attention_events
        attn = torch.empty(batch, n1, HEADS, head_dim, dtype=torch.bfloat16, device=x.device)
        attn_bhnd = attn.permute(0, 2, 1, 3)
        xr = x.view(rows, EMBED_DIM)
        h = add_layernorm(x, None, self.blocks[0].norm1.weight, self.blocks[0].norm1.bias, 1e-6)
        for layer, blk in enumerate(self.blocks):
            w_qkv, b_qkv, w_proj, _, w_fc1, _, w_fc2, _ = weights[layer]
            qkv = linear_bias(h, w_qkv, blk.attn.qkv.bias).view(batch, n1, 3, HEADS, head_dim)
            q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
            pose_l, fields_l = self._layer_look(values, layer)
            if self.attention_inputs is not None:
                kept = qkv.clone()
                self.attention_inputs.append(
                    tuple(kept[:, :, i].permute(0, 2, 1, 3) for i in range(3)) + (pose_l, fields_l, scale))
            if events is not None:
                start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
            look_attention_forward(q, k, v, pose_l, fields_l, scale=scale, out=attn_bhnd)
            if events is not None:
                stop.record()
                events.append((start, stop))
            h = linear_residual_layernorm(attn.view(rows, EMBED_DIM), w_proj, blk.attn.proj.bias, xr,
                                          blk.norm2.weight, blk.norm2.bias, 1e-6)
            u = linear_gelu(h, w_fc1, blk.mlp.fc1.bias)
            nxt = self.blocks[layer + 1].norm1 if layer + 1 < len(self.blocks) else self.norm
            h = linear_residual_layernorm(u, w_fc2, blk.mlp.fc2.bias, xr, nxt.weight, nxt.bias, 1e-6)
        h = h.view(batch, n1, EMBED_DIM)
        return h[:, 0] if cls_only else h

    def slot_fields(self) -> torch.Tensor:
        """F[h, p, s] = sum_g basis[p, g, s] * grid[h, g]: the Look field value of
        slot s for head h and pose p, (36, 12, S) fp32."""
        grid = self.look_bank.look_grid.float().reshape(LOOK_HEADS, -1)
        return torch.einsum("pgs,hg->hps", self.look_basis, grid)

    @torch.no_grad()
    def look_values(self, pose: torch.Tensor) -> torch.Tensor:
        """Per-query Look value of every slot, (B, N, 36, S) fp32 (pose @ F)."""
        return torch.einsum("bnhp,hps->bnhs", pose, self.slot_fields()).contiguous()

    def _trunk_weights(self, dtype):
        """Linear weights of the 12 blocks in the compute dtype (cached per weight version)."""
        if dtype == torch.float32:
            return [(b.attn.qkv.weight, b.attn.qkv.bias, b.attn.proj.weight, b.attn.proj.bias, b.mlp.fc1.weight,
                     b.mlp.fc1.bias, b.mlp.fc2.weight, b.mlp.fc2.bias) for b in self.blocks]
        key = ("trunk", dtype, tuple((p.data_ptr(), p._version) for p in self.blocks.parameters()))
        with self._cache_lock:
            hit = self._cache.get(key)
        if hit is None:
            hit = [tuple(t.detach().to(dtype) for t in (b.attn.qkv.weight, b.attn.qkv.bias, b.attn.proj.weight,
                                                         b.attn.proj.bias, b.mlp.fc1.weight, b.mlp.fc1.bias,
                                                         b.mlp.fc2.weight, b.mlp.fc2.bias)) for b in self.blocks]
            with self._cache_lock:
                self._cache = {k: v for k, v in self._cache.items() if k[0] != "trunk"}
                self._cache[key] = hit
        return hit

    @torch.no_grad()
    def trunk(self, tokens: torch.Tensor, attend) -> torch.Tensor:
        """CLS + position embedding, 12 blocks, final LayerNorm.  ``attend(layer,
        q, k, v, out)`` writes the attention output of one layer into ``out``, a
        (B, H, N, D) view of a token-major (B, N, H, D) buffer, and returns it."""
        cdt = torch.bfloat16 if self.precision == "bf16" else torch.float32
        batch, n = tokens.shape[0], self.num_patches
        weights = self._trunk_weights(cdt)
        head_dim = EMBED_DIM // HEADS
        attn_buf = torch.empty(batch, n + 1, HEADS, head_dim, dtype=cdt, device=tokens.device)
        x = torch.cat((self.cls_token.expand(batch, -1, -1), tokens), dim=1) + self.pos_embed
        for layer, blk in enumerate(self.blocks):
            w_qkv, b_qkv, w_proj, b_proj, w_fc1, b_fc1, w_fc2, b_fc2 = weights[layer]
            h = F.layer_norm(x, (EMBED_DIM,), blk.norm1.weight, blk.norm1.bias, 1e-6)
            qkv = F.linear(h.to(cdt), w_qkv, b_qkv)
            qkv = qkv.reshape(batch, n + 1, 3, HEADS, head_dim).permute(2, 0, 3, 1, 4)
            attn = attend(layer, qkv[0], qkv[1], qkv[2], attn_buf.permute(0, 2, 1, 3))
            attn = attn.transpose(1, 2).reshape(batch, n + 1, EMBED_DIM)
            x = x + F.linear(attn.to(cdt), w_proj, b_proj).float()
            h = F.layer_norm(x, (EMBED_DIM,), blk.norm2.weight, blk.norm2.bias, 1e-6)
            h = F.gelu(F.linear(h.to(cdt), w_fc1, b_fc1))
            x = x + F.linear(h, w_fc2, b_fc2).float()
        return F.layer_norm(x, (EMBED_DIM,), self.norm.weight, self.norm.bias, 1e-6)

    @torch.no_grad()
    def forward_features(self, image: torch.Tensor) -> torch.Tensor:
        """Normalised tokens (B, N+1, 192) fp32."""
        if self.precision == "bf16":
            x, values = self.embed_fused(image)
            return self.trunk_fused(x, values).float()
        tokens, pose = self.embed(image)
        values = self.look_values(pose)
        scale = 1.0 / math.sqrt(EMBED_DIM // HEADS)
        events = self.attention_events

        def attend(layer, q, k, v, out):
            pose_l = values[:, :, HEADS * layer:HEADS * (layer + 1)]
            if events is not None:
                start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
            out, _ = look_attention_forward(q, k, v, pose_l, self.look_slots, scale=scale, out=out)
            if events is not None:
                stop.record()
                events.append((start, stop))
            return out

        return self.trunk(tokens, attend)

    @torch.no_grad()
    def forward(self, image: torch.Tensor) -> torch.Tensor:
        if self.precision == "bf16":
            x, values = self.embed_fused(image)
            cls = self.trunk_fused(x, values, cls_only=True)
            return F.linear(cls.float(), self.head.weight, self.head.bias)
        return F.linear(self.forward_features(image)[:, 0], self.head.weight, self.head.bias)
