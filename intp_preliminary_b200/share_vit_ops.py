"""Python side of the fused SHARE-ViT steps around the Look attention
(C ABI in include/intp_share_vit.h, kernels in csrc/share_vit_ops.cu).

Each function validates its tensors, then launches one kernel of
``libintp_b200.so`` on the current stream.  There is no PyTorch fallback:
CPU tensors, wrong dtypes or layouts raise ``ValueError``.
"""

from __future__ import annotations

import ctypes
from typing import NamedTuple

import torch

from . import _lib


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else None)


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require(cond: bool, message: str) -> None:
    if not cond:
        raise ValueError(message)


class GatherPlan(NamedTuple):
    """Shared-memory plan of the patch gather (``svit_gather_plan``): patches in
    groups of ``group_patches``; each group's distinct 16-byte image units (4
    pixels, offset // 4), sorted, in ``stage_offset[stage_begin[g]:stage_begin[g + 1]]``
    (int32); ``local_index`` (N, F) int16, the pixel's float position among its
    group's staged units (4 * unit rank + offset % 4)."""

    stage_offset: torch.Tensor
    stage_begin: torch.Tensor
    local_index: torch.Tensor
    group_patches: int
    max_stage: int
    max_offset: int

    def to(self, device: torch.device | str) -> "GatherPlan":
        return self._replace(stage_offset=self.stage_offset.to(device), stage_begin=self.stage_begin.to(device),
                             local_index=self.local_index.to(device))


# int16 float positions: at most 8191 units of 16 bytes (128 KB of shared memory).
_MAX_STAGE = 8191


def gather_plan(pixel_index: torch.Tensor, group_patches: int = 6) -> GatherPlan:
    """Build the staged gather's plan from ``pixel_index`` (N, F) int32 (host
    work, once per patch geometry).  The result lives on ``pixel_index``'s device."""
    _require(pixel_index.dtype == torch.int32 and pixel_index.ndim == 2, "pixel_index must be an (N, F) int32 tensor")
    _require(group_patches > 0, "group_patches must be positive")
    index = pixel_index.detach().cpu().long()
    patches, features = index.shape
    _require(features % 8 == 0, "features must be a multiple of 8")
    _require(patches == 0 or int(index.min()) >= 0, "pixel_index must be non-negative")
    offsets, begin, local = [], [0], torch.empty(patches, features, dtype=torch.int16)
    for n0 in range(0, patches, group_patches):
        rows = index[n0:n0 + group_patches]
        units, rank = torch.unique(rows // 4, sorted=True, return_inverse=True)
        _require(units.numel() <= _MAX_STAGE, f"a group of {group_patches} patches reads {units.numel()} "
                 f"16-byte units (at most {_MAX_STAGE}); use smaller groups")
        offsets.append(units.to(torch.int32))
        begin.append(begin[-1] + units.numel())
        local[n0:n0 + group_patches] = (4 * rank + rows % 4).to(torch.int16)
    counts = [b - a for a, b in zip(begin[:-1], begin[1:])]
    stage_offset = torch.cat(offsets) if offsets else torch.zeros(0, dtype=torch.int32)
    device = pixel_index.device
    return GatherPlan(stage_offset.to(device), torch.tensor(begin, dtype=torch.int32, device=device),
                      local.to(device), group_patches, max(counts, default=0),
                      int(index.max()) if patches else -1)


def gather_patches(image: torch.Tensor, pixel_index: torch.Tensor, weight: torch.Tensor,
                   out: torch.Tensor | None = None, plan: GatherPlan | None = None) -> torch.Tensor:
    """``out[b*N + n, f] = bf16(image[b].flatten()[pixel_index[n, f]] * weight[f])``.

    image (B, C, H, W) float32 contiguous CUDA; pixel_index (N, F) int32;
    weight (F,) float32.  Returns (B*N, F) bf16.  With ``plan`` (from
    ``gather_plan(pixel_index)``) the gather runs through shared memory."""
    _require(image.is_cuda and image.dtype == torch.float32 and image.is_contiguous(),
             "image must be a contiguous float32 CUDA tensor")
    _require(pixel_index.dtype == torch.int32 and pixel_index.ndim == 2 and pixel_index.is_contiguous(),
             "pixel_index must be a contiguous (N, F) int32 tensor")
    _require(weight.dtype == torch.float32 and weight.ndim == 1 and weight.shape[0] == pixel_index.shape[1],
             "weight must be a float32 (F,) tensor")
    _require(pixel_index.device == image.device and weight.device == image.device, "tensors must share a device")
    batch = image.shape[0]
    patches, features = pixel_index.shape
    if out is None:
        out = torch.empty((batch * patches, features), dtype=torch.bfloat16, device=image.device)
    _require(out.shape == (batch * patches, features) and out.dtype == torch.bfloat16 and out.is_contiguous(),
             "out must be a contiguous (B*N, F) bf16 tensor")
    image_elems = image[0].numel() if batch else 0
    if plan is None:
        status = _lib.load().svit_gather_patches(
            _ptr(image), batch, image_elems, _ptr(pixel_index), _ptr(weight), patches, features,
            _ptr(out), _stream(image.device))
    else:
        _require(plan.local_index.shape == (patches, features) and plan.local_index.dtype == torch.int16
                 and plan.local_index.is_contiguous(), "plan does not match pixel_index")
        _require(all(t.device == image.device for t in (plan.stage_offset, plan.stage_begin, plan.local_index)),
                 "plan must be on the image's device")
        _require(batch == 0 or (plan.max_offset < image_elems and image_elems % 4 == 0),
                 "plan reads beyond one image, or images are not whole 16-byte units")
        groups = plan.stage_begin.numel() - 1
        args = _lib.SvitGatherPlan(_ptr(plan.stage_offset).value, _ptr(plan.stage_begin).value,
                                   _ptr(plan.local_index).value, groups, plan.group_patches, plan.max_stage)
        status = _lib.load().svit_gather_patches_staged(
            _ptr(image), batch, image_elems, ctypes.byref(args), _ptr(weight), patches, features, _ptr(out),
            _stream(image.device))
    _lib.check(status, "hex patch gather")
    return out


def embed_post(resp: torch.Tensor, *, batch: int, patches: int, bases: int, directions: int, look_heads: int,
               look_poses: int, token_null: torch.Tensor, direction_coef: torch.Tensor, output_bias: torch.Tensor,
               cls: torch.Tensor, pos_embed: torch.Tensor, look_null: torch.Tensor, slot_fields: torch.Tensor,
               x: torch.Tensor, values: torch.Tensor | None, look_pose: torch.Tensor | None = None) -> None:
    """Tokens (with CLS and position embedding) into ``x`` (B, N+1, 2*bases),
    per-slot Look values into ``values`` (B, look_heads, N, slots) and / or
    the Look pose into ``look_pose`` (B, N, look_heads, look_poses), from the
    bf16 response rows ``resp`` (B*N, >= bases*directions + look_poses*look_heads).
    With ``values=None`` the per-slot products are left to the attention
    (``LookSlotFields``)."""
    dev = resp.device
    _require(resp.is_cuda and resp.dtype == torch.bfloat16 and resp.ndim == 2 and resp.stride(1) == 1,
             "resp must be a bf16 CUDA matrix with unit column stride")
    _require(resp.shape[0] == batch * patches, "resp must have batch * patches rows")
    _require(values is not None or look_pose is not None, "values or look_pose is needed")
    fp32 = [t for t in (token_null, direction_coef, output_bias, cls, pos_embed, look_null, slot_fields, x, values,
                        look_pose) if t is not None]
    for t in fp32:
        _require(t.device == dev and t.dtype == torch.float32 and t.is_contiguous(),
                 "parameters and outputs must be contiguous float32 tensors on resp's device")
    slots = slot_fields.shape[-1]
    _require(slot_fields.shape == (look_heads, look_poses, slots), "slot_fields must be (look_heads, look_poses, S)")
    _require(x.shape == (batch, patches + 1, 2 * bases), "x must be (B, N+1, 2*bases)")
    _require(values is None or values.shape == (batch, look_heads, patches, slots),
             "values must be (B, look_heads, N, S)")
    _require(look_pose is None or look_pose.shape == (batch, patches, look_heads, look_poses),
             "look_pose must be (B, N, look_heads, look_poses)")
    a = _lib.SvitEmbedArgs()
    a.batch, a.patches = batch, patches
    a.bases, a.directions, a.look_heads, a.look_poses, a.slots = bases, directions, look_heads, look_poses, slots
    a.resp, a.resp_stride = resp.data_ptr(), resp.stride(0)
    a.token_null, a.direction_coef, a.output_bias = token_null.data_ptr(), direction_coef.data_ptr(), output_bias.data_ptr()
    a.cls, a.pos_embed, a.look_null, a.slot_fields = cls.data_ptr(), pos_embed.data_ptr(), look_null.data_ptr(), slot_fields.data_ptr()
    a.x = x.data_ptr()
    a.values = values.data_ptr() if values is not None else None
    a.look_pose = look_pose.data_ptr() if look_pose is not None else None
    status = _lib.load().svit_embed_post(ctypes.byref(a), _stream(dev))
    _lib.check(status, "tokenizer / Look-bank post-processing")


def tokenizer_gemm(patches: torch.Tensor, weight: torch.Tensor, *, batch: int, patches_per_image: int, bases: int,
                   directions: int, look_heads: int, look_poses: int, token_null: torch.Tensor,
                   direction_coef: torch.Tensor, output_bias: torch.Tensor, cls: torch.Tensor, pos_embed: torch.Tensor,
                   look_null: torch.Tensor, x: torch.Tensor, look_pose: torch.Tensor) -> None:
    """The tokenizer + Look-bank GEMM with ``embed_post``'s softmaxes in its
    epilogue (one tcgen05 kernel; the response matrix is never stored):
    tokens into ``x`` (B, N+1, 2*bases) and the Look pose into ``look_pose``
    (B, N, look_heads, look_poses) from the bf16 ``patches`` (B*N, F) and the
    bf16 ``weight`` (bases*directions + look_heads*look_poses, F) whose Look
    rows are ordered head by head."""
    dev = patches.device
    _require(patches.is_cuda and patches.dtype == torch.bfloat16 and patches.ndim == 2 and patches.stride(1) == 1,
             "patches must be a bf16 CUDA matrix with unit column stride")
    _require(patches.shape[0] == batch * patches_per_image, "patches must have batch * patches_per_image rows")
    rows_w = bases * directions + look_heads * look_poses
    _require(weight.device == dev and weight.dtype == torch.bfloat16 and weight.is_contiguous()
             and tuple(weight.shape) == (rows_w, patches.shape[1]),
             "weight must be a contiguous bf16 (bases*directions + look_heads*look_poses, F) matrix")
    for t in (token_null, direction_coef, output_bias, cls, pos_embed, look_null, x, look_pose):
        _require(t.device == dev and t.dtype == torch.float32 and t.is_contiguous(),
                 "parameters and outputs must be contiguous float32 tensors on the patches' device")
    _require(x.shape == (batch, patches_per_image + 1, 2 * bases), "x must be (B, N+1, 2*bases)")
    _require(look_pose.shape == (batch, patches_per_image, look_heads, look_poses),
             "look_pose must be (B, N, look_heads, look_poses)")
    a = _lib.SvitEmbedArgs()
    a.batch, a.patches = batch, patches_per_image
    a.bases, a.directions, a.look_heads, a.look_poses, a.slots = bases, directions, look_heads, look_poses, 0
    a.token_null, a.direction_coef, a.output_bias = token_null.data_ptr(), direction_coef.data_ptr(), output_bias.data_ptr()
    a.cls, a.pos_embed, a.look_null = cls.data_ptr(), pos_embed.data_ptr(), look_null.data_ptr()
    a.x, a.values, a.look_pose = x.data_ptr(), None, look_pose.data_ptr()
    status = _lib.load().svit_tokenizer_gemm(ctypes.byref(a), ctypes.c_void_p(patches.data_ptr()), patches.stride(0),
                                             patches.shape[1], ctypes.c_void_p(weight.data_ptr()),
                                             _status(dev), _stream(dev))
    _lib.check(status, "fused tokenizer / Look-bank GEMM")


def add_layernorm(x: torch.Tensor, y: torch.Tensor | None, weight: torch.Tensor, bias: torch.Tensor, eps: float,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """``x += y`` (when given, in place) then ``out = bf16(LayerNorm(x))`` over the last dim.

    x float32 (..., dim) with unit last stride and rows at a common stride;
    y bf16 of the same row shape or None."""
    dim = x.shape[-1]
    _require(x.is_cuda and x.dtype == torch.float32 and x.stride(-1) == 1, "x must be float32 CUDA, unit last stride")
    xr = x.reshape(-1, dim)
    _require(xr.data_ptr() == x.data_ptr(), "x rows must be addressable with one stride")
    rows = xr.shape[0]
    if y is not None:
        _require(y.dtype == torch.bfloat16 and y.device == x.device and y.shape[-1] == dim, "y must be bf16 like x")
        yr = y.reshape(-1, dim)
        _require(yr.shape[0] == rows and yr.stride(-1) == 1, "y must match x's rows")
    else:
        yr = None
    for t in (weight, bias):
        _require(t.dtype == torch.float32 and t.is_contiguous() and t.shape == (dim,) and t.device == x.device,
                 "LayerNorm weight and bias must be contiguous float32 (dim,)")
    if out is None:
        out = torch.empty((rows, dim), dtype=torch.bfloat16, device=x.device)
    outr = out.reshape(-1, dim)
    _require(out.dtype == torch.bfloat16 and outr.shape[0] == rows and outr.stride(-1) == 1, "out must be bf16 rows")
    status = _lib.load().svit_add_layernorm(
        _ptr(xr), xr.stride(0), _ptr(yr), yr.stride(0) if yr is not None else 0, _ptr(weight), _ptr(bias),
        float(eps), rows, dim, _ptr(outr), outr.stride(0), _stream(x.device))
    _lib.check(status, "add + LayerNorm")
    return out


def _linear_checks(a: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    _require(a.is_cuda and a.dtype == torch.bfloat16 and a.ndim == 2 and a.stride(1) == 1,
             "input must be a bf16 CUDA matrix with unit column stride")
    _require(weight.dtype == torch.bfloat16 and weight.is_contiguous() and weight.ndim == 2
             and weight.shape[1] == a.shape[1] and weight.device == a.device,
             "weight must be a contiguous bf16 (out_features, in_features) tensor on the input's device")
    _require(bias.dtype == torch.float32 and bias.is_contiguous() and bias.shape == (weight.shape[0],)
             and bias.device == a.device, "bias must be a contiguous float32 (out_features,) tensor")
    _require(a.shape[1] % 64 == 0, "in_features must be a multiple of 64")
    return a


def _status(device: torch.device) -> ctypes.c_void_p:
    from .look_attention import _status_word

    return ctypes.c_void_p(_status_word(device).data_ptr())


def linear_gelu(a: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """``bf16(GELU(a @ weight.T + bias))`` (exact erf GELU) on the tcgen05 GEMM with
    the activation in its epilogue.  a (rows, K) bf16, weight (N, K) bf16, bias (N,) fp32."""
    _linear_checks(a, weight, bias)
    rows, k = a.shape
    n = weight.shape[0]
    _require(n % 256 == 0, "out_features must be a multiple of 256")
    out = torch.empty(rows, n, dtype=torch.bfloat16, device=a.device)
    status = _lib.load().svit_linear_gelu(_ptr(a), a.stride(0), rows, k, _ptr(weight), _ptr(bias), n, _ptr(out),
                                          out.stride(0), _status(a.device), _stream(a.device))
    _lib.check(status, "linear + GELU")
    return out


def linear_bias(a: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """``bf16(a @ weight.T + bias)`` on the tcgen05 GEMM (the attention's qkv
    projection).  a (rows, K) bf16, weight (N, K) bf16 with N % 192 == 0, bias (N,) fp32."""
    _linear_checks(a, weight, bias)
    rows, k = a.shape
    n = weight.shape[0]
    _require(n % 192 == 0, "out_features must be a multiple of 192")
    out = torch.empty(rows, n, dtype=torch.bfloat16, device=a.device)
    status = _lib.load().svit_linear_bias(_ptr(a), a.stride(0), rows, k, _ptr(weight), _ptr(bias), n, _ptr(out),
                                          out.stride(0), _status(a.device), _stream(a.device))
    _lib.check(status, "linear + bias")
    return out


def linear_residual_layernorm(a: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, x: torch.Tensor,
                              norm_weight: torch.Tensor, norm_bias: torch.Tensor, eps: float) -> torch.Tensor:
    """``x += a @ weight.T + bias`` (x float32, in place) and return
    ``bf16(LayerNorm(x))``, from one tcgen05 GEMM with the residual add and the
    LayerNorm in its epilogue.  dim = weight.shape[0] = 192."""
    _linear_checks(a, weight, bias)
    rows, k = a.shape
    dim = weight.shape[0]
    _require(x.dtype == torch.float32 and x.device == a.device and x.shape[-1] == dim and x.stride(-1) == 1,
             "x must be float32 with unit last stride and dim columns")
    xr = x.reshape(-1, dim)
    _require(xr.data_ptr() == x.data_ptr() and xr.shape[0] == rows, "x rows must match the input rows")
    for t in (norm_weight, norm_bias):
        _require(t.dtype == torch.float32 and t.is_contiguous() and t.shape == (dim,) and t.device == a.device,
                 "LayerNorm weight and bias must be contiguous float32 (dim,)")
    h = torch.empty(rows, dim, dtype=torch.bfloat16, device=a.device)
    status = _lib.load().svit_linear_residual_layernorm(
        _ptr(a), a.stride(0), rows, k, _ptr(weight), _ptr(bias), dim, _ptr(xr), xr.stride(0), _ptr(norm_weight),
        _ptr(norm_bias), float(eps), _ptr(h), h.stride(0), _status(a.device), _stream(a.device))
    _lib.check(status, "linear + residual + LayerNorm")
    return h


def _time_block_linears(batch: int = 256, steps: int = 20) -> dict[str, float]:
    """The transformer block's three fused linears at the half6d3r shapes
    (batch x 197 token rows, 192 / 768 features, seeded inputs): 3 warm-up
    calls each, one more call each (the launches a profiler captures with
    ``-s 9 -c 3``), then ``steps`` calls each timed with CUDA events.
    Returns microseconds per call."""
    dev = torch.device("cuda", torch.cuda.current_device())
    rows = batch * 197
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randn(rows, 192, device=dev, generator=g).to(torch.bfloat16)
    a2 = torch.randn(rows, 768, device=dev, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(768, 192, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    b1 = torch.randn(768, device=dev, generator=g) * 0.1
    wp = (torch.randn(192, 192, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(192, 768, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    bp = torch.randn(192, device=dev, generator=g) * 0.1
    x = torch.randn(rows, 192, device=dev, generator=g)
    gamma = torch.rand(192, device=dev, generator=g) + 0.5
    beta = torch.randn(192, device=dev, generator=g) * 0.1
    calls = {
        "fc1 + GELU (K 192, N 768)": lambda: linear_gelu(a, w1, b1),
        "proj + residual + LayerNorm (K 192, N 192)": lambda: linear_residual_layernorm(a, wp, bp, x, gamma, beta,
                                                                                       1e-6),
        "fc2 + residual + LayerNorm (K 768, N 192)": lambda: linear_residual_layernorm(a2, w2, bp, x, gamma, beta,
                                                                                      1e-6),
    }
    for _ in range(4):
        for fn in calls.values():
            fn()
    torch.cuda.synchronize()
    result = {}
    for name, fn in calls.items():
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            fn()
        stop.record()
        torch.cuda.synchronize()
        result[name] = start.elapsed_time(stop) / steps * 1000.0
    return result


def _time_patch_gather(batch: int = 256, steps: int = 20) -> dict[str, float]:
    """The half6d3r patch gather (batch seeded 224 x 224 x 3 images, the model's
    (195, 1680) pixel table), direct and staged: 3 warm-up calls each (the
    staged launches a profiler skips with ``-s 3``), then ``steps`` calls each,
    every call timed alone with CUDA events after a 256 MB write that flushes
    the L2.  Returns the median microseconds per call."""
    from .share_vit import ShareViTHalf6d3r
    dev = torch.device("cuda", torch.cuda.current_device())
    model = ShareViTHalf6d3r().to(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    images = torch.randn(batch, 3, 224, 224, device=dev, generator=g)
    out = torch.empty(batch * model.num_patches, model.pixel_index.shape[1], dtype=torch.bfloat16, device=dev)
    plan = GatherPlan(model.gather_stage_offset, model.gather_stage_begin, model.gather_local_index,
                      *model._gather_plan_sizes)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    calls = {
        "staged (shared-memory plan)": lambda: gather_patches(images, model.pixel_index, model.pixel_weight, out,
                                                              plan=plan),
        "direct": lambda: gather_patches(images, model.pixel_index, model.pixel_weight, out),
    }
    result = {}
    for name, fn in calls.items():
        for _ in range(3):
            fn()
        times = []
        for _ in range(steps):
            flush.fill_(1)
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            fn()
            stop.record()
            torch.cuda.synchronize()
            times.append(start.elapsed_time(stop) * 1000.0)
        result[name] = sorted(times)[len(times) // 2]
    return result


if __name__ == "__main__":
    import sys
    runner = _time_patch_gather if sys.argv[1:] == ["gather"] else _time_block_linears
    for name, us in runner().items():
        print(f"{name}: {us:.1f} us")
