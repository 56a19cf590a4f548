"""Fused SHARE-ViT kernels (gather, post-GEMM, add + LayerNorm) against the
plain PyTorch formulation of the same steps."""

import math

import pytest
import torch
import torch.nn.functional as F

from intp_preliminary_b200 import share_vit_ops as ops
from intp_preliminary_b200.share_vit import EMBED_DIM, LookPose, ShareViTHalf6d3r

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(cuda_device):
    return ShareViTHalf6d3r(precision="bf16").init_weights(seed=1, look_grid_std=0.5).to(cuda_device)


def test_gather_patches_matches_reflect_gather(model, cuda_device):
    images = torch.randn(3, 3, 224, 224, device=cuda_device, generator=torch.Generator(cuda_device).manual_seed(2))
    got = ops.gather_patches(images, model.pixel_index, model.pixel_weight)
    ref = torch.cat([model._patches(images, 0), model._patches(images, 1)], dim=-1).reshape(3 * 195, -1)
    assert torch.equal(got, ref.to(torch.bfloat16))


@pytest.mark.parametrize("group_patches", [1, 5, 8, 13, 26])
def test_staged_gather_equals_direct_gather(model, cuda_device, group_patches):
    """The shared-memory gather is bit-exact with the direct one on the model's
    geometry, for any grouping (partial last groups, up to 26 patches per group)."""
    images = torch.randn(5, 3, 224, 224, device=cuda_device, generator=torch.Generator(cuda_device).manual_seed(3))
    plan = ops.gather_plan(model.pixel_index, group_patches)
    got = ops.gather_patches(images, model.pixel_index, model.pixel_weight, plan=plan)
    assert torch.equal(got, ops.gather_patches(images, model.pixel_index, model.pixel_weight))


def test_staged_gather_random_geometry(cuda_device):
    """Arbitrary offsets (repeats, unsorted, touching the image's last element)."""
    g = torch.Generator().manual_seed(4)
    images = torch.randn(3, 2, 9, 12, generator=g).to(cuda_device)
    index = torch.randint(0, 2 * 9 * 12, (37, 64), generator=g, dtype=torch.int32)
    index[5, 7] = 2 * 9 * 12 - 1
    weight = torch.randn(64, generator=g)
    index, weight = index.to(cuda_device), weight.to(cuda_device)
    ref = (images.reshape(3, -1)[:, index.long()] * weight).reshape(3 * 37, 64).to(torch.bfloat16)
    for group in (1, 4, 37):
        got = ops.gather_patches(images, index, weight, plan=ops.gather_plan(index, group))
        assert torch.equal(got, ref)


def test_model_embed_uses_staged_gather(model, cuda_device):
    """The model's registered plan is the one gather_plan builds."""
    plan = ops.gather_plan(model.pixel_index, model._gather_plan_sizes[0])
    assert (plan.group_patches, plan.max_stage, plan.max_offset) == model._gather_plan_sizes
    assert torch.equal(model.gather_stage_offset, plan.stage_offset)
    assert torch.equal(model.gather_local_index, plan.local_index)
    assert model.gather_stage_offset.device == model.pixel_index.device


@pytest.mark.parametrize("rows,dim", [(1, 192), (37, 192), (50432 // 16, 192), (9, 64), (5, 512)])
def test_add_layernorm_matches_torch(cuda_device, rows, dim):
    g = torch.Generator(cuda_device).manual_seed(rows)
    x = torch.randn(rows, dim, device=cuda_device, generator=g) * 3 + 1
    y = torch.randn(rows, dim, device=cuda_device, generator=g).to(torch.bfloat16)
    w = torch.randn(dim, device=cuda_device, generator=g)
    b = torch.randn(dim, device=cuda_device, generator=g)
    x_ref = x + y.float()
    h_ref = F.layer_norm(x_ref, (dim,), w, b, 1e-6)
    h = ops.add_layernorm(x, y, w, b, 1e-6)
    assert torch.equal(x, x_ref)
    torch.testing.assert_close(h.float(), h_ref, atol=3e-2, rtol=1e-2)
    assert (h.float() - h_ref.to(torch.bfloat16).float()).abs().max() <= 2 * 2 ** -8 * h_ref.abs().max()
    h2 = ops.add_layernorm(x, None, w, b, 1e-6)
    torch.testing.assert_close(h2.float(), h_ref, atol=3e-2, rtol=1e-2)


def test_add_layernorm_on_strided_rows(cuda_device):
    x = torch.randn(4, 7, 192, device=cuda_device)
    y = torch.randn(4, 7, 192, device=cuda_device).to(torch.bfloat16)
    w, b = torch.ones(192, device=cuda_device), torch.zeros(192, device=cuda_device)
    x0 = x.clone()
    h = ops.add_layernorm(x[:, 0], y[:, 0], w, b, 1e-6)
    ref = F.layer_norm(x0[:, 0] + y[:, 0].float(), (192,), w, b, 1e-6)
    torch.testing.assert_close(h.float(), ref, atol=3e-2, rtol=1e-2)
    assert torch.equal(x[:, 1:], x0[:, 1:])


def test_embed_fused_matches_unfused(model, cuda_device):
    images = torch.randn(4, 3, 224, 224, device=cuda_device, generator=torch.Generator(cuda_device).manual_seed(3))
    x, values = model.embed_fused(images, per_slot_values=True)
    tokens, pose = model.embed(images)
    ref_values = model.look_values(pose)
    ref_x = torch.cat((model.cls_token.expand(4, -1, -1), tokens), dim=1) + model.pos_embed
    torch.testing.assert_close(x, ref_x, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(values, ref_values, atol=3e-2, rtol=3e-2)
    assert torch.equal(x[:, 0], (model.cls_token[0, 0] + model.pos_embed[0, 0]).expand(4, -1))
    # default: the Look pose and slot values instead of their product, from the
    # fused tokenizer GEMM (fp32 scores instead of the bf16 response matrix)
    x2, look = model.embed_fused(images)
    assert isinstance(look, LookPose)
    torch.testing.assert_close(x2, ref_x, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(look.pose, pose, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(look.fields, model.slot_fields(), atol=1e-6, rtol=1e-5)
    x3, look3 = model.embed_fused(images, fused_tokenizer=False)
    torch.testing.assert_close(x3, x, atol=0, rtol=0)


@pytest.mark.parametrize("batch", [3, 5, 64])
def test_tokenizer_gemm_matches_float64_and_unfused(model, cuda_device, batch):
    """The fused tokenizer GEMM (one tcgen05 kernel, softmaxes from the fp32
    accumulators) against the float64 computation on the same bf16 patches and
    weights, and against the cuBLAS GEMM + embed_post path (bf16 response)
    within that path's rounding.  256-row tiles of two 128-row halves: 3 images
    = 585 rows (the last tile's second half wholly past the end), 5 images =
    975 rows (a partial second half), 64 images = 12480 rows (343 tiles: CTAs
    take up to three tiles through the single accumulator); K = 1680: a
    partial last K slab."""
    n = model.num_patches
    images = torch.randn(batch, 3, 224, 224, device=cuda_device, generator=torch.Generator(cuda_device).manual_seed(21))
    patches = ops.gather_patches(images, model.pixel_index, model.pixel_weight)
    wt, _ = model._tokenizer_weights(cuda_device)
    params = dict(token_null=model.patch_embed.null_score.detach().float().contiguous(),
                  direction_coef=model.direction_coefficients.contiguous(),
                  output_bias=model.patch_embed.output_bias.detach().float().contiguous(),
                  cls=model.cls_token.detach().float().reshape(-1).contiguous(),
                  pos_embed=model.pos_embed.detach().float().reshape(n + 1, EMBED_DIM).contiguous(),
                  look_null=model.look_bank.null_score.detach().float().contiguous())
    x = torch.full((batch, n + 1, EMBED_DIM), float("nan"), device=cuda_device)
    pose = torch.full((batch, n, 36, 12), float("nan"), device=cuda_device)
    ops.tokenizer_gemm(patches, wt, batch=batch, patches_per_image=n, bases=96, directions=6, look_heads=36,
                       look_poses=12, x=x, look_pose=pose, **params)
    resp = patches.double() @ wt.double().T
    tok = resp[:, :576].reshape(batch, n, 96, 6)
    tnull = params["token_null"].double()[None, None, :, None].expand(batch, n, 96, 1)
    w = torch.cat((tok, tnull), -1).softmax(-1)[..., :-1]
    tokens = torch.einsum("bnpd,dc->bnpc", w, params["direction_coef"].double()).reshape(batch, n, EMBED_DIM)
    tokens = tokens + params["output_bias"].double()
    ref_x = torch.cat((params["cls"].double().expand(batch, 1, -1), tokens), dim=1) + params["pos_embed"].double()
    look = resp[:, 576:].reshape(batch, n, 36, 12)
    lnull = params["look_null"].double()[None, None, :, None].expand(batch, n, 36, 1)
    ref_pose = torch.cat((look, lnull), -1).softmax(-1)[..., :-1]
    assert (x.double() - ref_x).abs().max().item() <= 1e-4
    assert (pose.double() - ref_pose).abs().max().item() <= 1e-5
    x_old, look_old = model.embed_fused(images, fused_tokenizer=False)
    torch.testing.assert_close(x, x_old, atol=2e-2, rtol=0)
    torch.testing.assert_close(pose, look_old.pose, atol=1e-2, rtol=0)


@pytest.mark.parametrize("features", [200, 1680])
def test_tokenizer_gemm_other_shapes(cuda_device, features):
    """Shapes other than the model's: 48 bases (two tokenizer tiles), 12 Look
    heads (one Look tile), 50 patches per image, 3 images = 150 rows (one
    partial 256-row tile whose second half is short), random operands; the
    float64 computation on the same bf16 values is the reference."""
    gen = torch.Generator().manual_seed(31)
    batch, n, bases, heads = 3, 50, 48, 12
    dim = 2 * bases
    patches = (torch.randn(batch * n, features, generator=gen) / 4).to(torch.bfloat16)
    weight = (torch.randn(6 * bases + 12 * heads, features, generator=gen) / 4).to(torch.bfloat16)
    p = dict(token_null=torch.randn(bases, generator=gen), direction_coef=torch.randn(6, 2, generator=gen),
             output_bias=torch.randn(dim, generator=gen), cls=torch.randn(dim, generator=gen),
             pos_embed=torch.randn(n + 1, dim, generator=gen), look_null=torch.randn(heads, generator=gen))
    dev = {k: v.to(cuda_device) for k, v in p.items()}
    x = torch.full((batch, n + 1, dim), float("nan"), device=cuda_device)
    pose = torch.full((batch, n, heads, 12), float("nan"), device=cuda_device)
    ops.tokenizer_gemm(patches.to(cuda_device), weight.to(cuda_device), batch=batch, patches_per_image=n,
                       bases=bases, directions=6, look_heads=heads, look_poses=12, x=x, look_pose=pose, **dev)
    resp = patches.double() @ weight.double().T
    tok = resp[:, :6 * bases].reshape(batch, n, bases, 6)
    tnull = p["token_null"].double()[None, None, :, None].expand(batch, n, bases, 1)
    w = torch.cat((tok, tnull), -1).softmax(-1)[..., :-1]
    tokens = torch.einsum("bnpd,dc->bnpc", w, p["direction_coef"].double()).reshape(batch, n, dim)
    ref_x = torch.cat((p["cls"].double().expand(batch, 1, -1), tokens + p["output_bias"].double()), dim=1)
    ref_x = ref_x + p["pos_embed"].double()
    look = resp[:, 6 * bases:].reshape(batch, n, heads, 12)
    lnull = p["look_null"].double()[None, None, :, None].expand(batch, n, heads, 1)
    ref_pose = torch.cat((look, lnull), -1).softmax(-1)[..., :-1]
    assert (x.cpu().double() - ref_x).abs().max().item() <= 1e-4
    assert (pose.cpu().double() - ref_pose).abs().max().item() <= 1e-5


def test_tokenizer_gemm_rejects_what_it_cannot_take(model, cuda_device):
    n = model.num_patches
    patches = torch.zeros(2 * n, 1680, dtype=torch.bfloat16, device=cuda_device)
    wt, _ = model._tokenizer_weights(cuda_device)
    z = lambda *s: torch.zeros(*s, device=cuda_device)  # noqa: E731
    kw = dict(token_null=z(96), direction_coef=z(6, 2), output_bias=z(192), cls=z(192), pos_embed=z(n + 1, 192),
              look_null=z(36), x=z(2, n + 1, 192), look_pose=z(2, n, 36, 12))
    with pytest.raises(ValueError):
        ops.tokenizer_gemm(patches, wt[:-1], batch=2, patches_per_image=n, bases=96, directions=6, look_heads=36,
                           look_poses=12, **kw)
    with pytest.raises(RuntimeError):  # 10 bases: not a multiple of the kernel's 24-base tile
        ops.tokenizer_gemm(patches, wt[: 60 + 432], batch=2, patches_per_image=n, bases=10, directions=6,
                           look_heads=36, look_poses=12, **{**kw, "x": z(2, n + 1, 20), "output_bias": z(20),
                                                            "cls": z(20), "pos_embed": z(n + 1, 20),
                                                            "token_null": z(10)})


def test_look_pose_trunk_matches_per_slot_values(model, cuda_device):
    """The attention forming pose . slot values itself (SLOT_FIELDS) gives the
    trunk of the per-slot-values (SLOTS) path."""
    images = torch.randn(5, 3, 224, 224, device=cuda_device, generator=torch.Generator(cuda_device).manual_seed(12))
    x1, look = model.embed_fused(images)
    x2, values = model.embed_fused(images, per_slot_values=True)
    a = model.trunk_fused(x1, look).float()
    b = model.trunk_fused(x2, values).float()
    err = (a - b).abs().max().item()
    assert err <= 2e-2 * b.abs().max().item(), err


def test_fused_forward_matches_unfused_bf16(model, cuda_device):
    images = torch.randn(6, 3, 224, 224, device=cuda_device, generator=torch.Generator(cuda_device).manual_seed(4))
    fused = model(images)
    tokens, pose = model.embed(images)
    values = model.look_values(pose)
    scale = 1.0 / math.sqrt(64)
    from intp_preliminary_b200.look_attention import look_attention_forward

    def attend(layer, q, k, v, out):
        return look_attention_forward(q, k, v, values[:, :, 3 * layer:3 * layer + 3], model.look_slots, scale=scale,
                                      out=out)[0]

    feats = model.trunk(tokens, attend)
    ref = F.linear(feats[:, 0], model.head.weight, model.head.bias)
    err = (fused - ref).abs().max().item()
    assert err <= 0.05 * ref.abs().max().item(), err
    assert fused.shape == (6, 100) and torch.isfinite(fused).all()
    feats_fused = model.forward_features(images)
    assert feats_fused.shape == (6, 196, EMBED_DIM)


@pytest.mark.parametrize("rows", [1, 130, 4096 + 77])
def test_linear_gelu_matches_torch(cuda_device, rows):
    g = torch.Generator(cuda_device).manual_seed(rows)
    a = (torch.randn(rows, 192, device=cuda_device, generator=g)).to(torch.bfloat16)
    w = (torch.randn(768, 192, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
    b = torch.randn(768, device=cuda_device, generator=g) * 0.1
    out = ops.linear_gelu(a, w, b)
    ref = F.gelu(a.float() @ w.float().t() + b)
    assert out.dtype == torch.bfloat16 and out.shape == (rows, 768)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("rows,n", [(1, 576), (130, 192), (4096 + 77, 576)])
def test_linear_bias_matches_torch(cuda_device, rows, n):
    g = torch.Generator(cuda_device).manual_seed(rows + n)
    a = torch.randn(rows, 192, device=cuda_device, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, 192, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
    b = torch.randn(n, device=cuda_device, generator=g) * 0.1
    out = ops.linear_bias(a, w, b)
    ref = a.float() @ w.float().t() + b
    assert out.dtype == torch.bfloat16 and out.shape == (rows, n)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("rows,k", [(1, 192), (130, 192), (4096 + 77, 768)])
def test_linear_residual_layernorm_matches_torch(cuda_device, rows, k):
    g = torch.Generator(cuda_device).manual_seed(rows + k)
    a = torch.randn(rows, k, device=cuda_device, generator=g).to(torch.bfloat16)
    w = (torch.randn(192, k, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
    b = torch.randn(192, device=cuda_device, generator=g) * 0.1
    x = torch.randn(rows, 192, device=cuda_device, generator=g)
    nw = torch.randn(192, device=cuda_device, generator=g)
    nb = torch.randn(192, device=cuda_device, generator=g)
    x_ref = x + (a.float() @ w.float().t() + b)
    h_ref = F.layer_norm(x_ref, (192,), nw, nb, 1e-6)
    h = ops.linear_residual_layernorm(a, w, b, x, nw, nb, 1e-6)
    torch.testing.assert_close(x, x_ref, atol=1e-3, rtol=1e-4)
    torch.testing.assert_close(h.float(), h_ref, atol=3e-2, rtol=1e-2)


def test_tcgen05_linears_match_cublas_trunk(model, cuda_device):
    images = torch.randn(5, 3, 224, 224, device=cuda_device, generator=torch.Generator(cuda_device).manual_seed(11))
    x1, values = model.embed_fused(images)
    x2 = x1.clone()
    fused = model.trunk_fused(x1, values, linears="tcgen05").float()
    plain = model.trunk_fused(x2, values, linears="cublas").float()
    err = (fused - plain).abs().max().item()
    assert err <= 5e-2 * plain.abs().max().item(), err
    assert torch.isfinite(fused).all()

