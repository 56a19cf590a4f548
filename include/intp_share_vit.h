/*
 * intp_share_vit.h - C ABI of the fused steps of the half6d3r SHARE-ViT
 * forward that surround the Look attention (libintp_b200.so).
 *
 * The reference runs these steps as chains of PyTorch operators; each entry
 * point below replaces one such chain with one kernel:
 *   svit_gather_patches : HexPatchGeometry's reflect-padded circular gather
 *                         and the cover weighting of both supports
 *                         (layers/hex_patch_geometry.py:82-90,
 *                          layers/rotating_dot_product.py:9-13), cast to bf16
 *                         as the input of the tokenizer / Look-bank GEMM.
 *   svit_embed_post     : after that GEMM, the tokenizer's null softmax and
 *                         harmonic moments (layers/hex_rotating_harmonic_patch_embed.py:153-242),
 *                         CLS + position embedding
 *                         (model/deit_tiny_rot_hex_look.py:305-452), and the
 *                         Look bank's null softmax (layers/square_patch_dense_grid_look.py:339-355)
 *                         contracted with the per-slot Look fields into the
 *                         per-query Look values the attention kernel reads.
 *   svit_tokenizer_gemm : that GEMM with svit_embed_post's softmaxes in its
 *                         epilogue (tcgen05; the response matrix is never stored).
 *   svit_add_layernorm  : residual add + LayerNorm + bf16 cast of the
 *                         pre-norm transformer block (layers/mini_vit.py:138-170).
 *   svit_linear_gelu,   : the block's linear layers on tcgen05 with GELU, or
 *   svit_linear_residual_layernorm   residual add + next LayerNorm, in the epilogue.
 * Same conventions as intp_b200.h: device pointers, element strides, a CUDA
 * stream, intp_status return codes; nothing is allocated or freed.
 */
#ifndef INTP_SHARE_VIT_H
#define INTP_SHARE_VIT_H

#include <stdint.h>
#include "intp_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* out[b * patches + n, f] = bf16(image[b][pixel_index[n, f]] * weight[f])
 * image: (batch, image_elems) float32 contiguous; pixel_index: (patches,
 * features) int32 offsets into one image (already reflected into range);
 * weight: (features) float32; out: (batch * patches, features) bf16,
 * row-major.  features % 8 == 0.                                            */
INTP_API intp_status svit_gather_patches(const float* image, int64_t batch, int64_t image_elems,
                                         const int32_t* pixel_index, const float* weight, int64_t patches,
                                         int64_t features, void* out, void* stream);

/* The same gather through shared memory.  Patches are taken in groups of
 * group_patches consecutive ones (the last group may hold fewer); the 16-byte
 * image units (4 pixels; unit u holds offsets 4u .. 4u + 3) that a group
 * reads are listed once, sorted, in stage_offset[stage_begin[g] ..
 * stage_begin[g + 1]), and local_index[n, f] is the float position of
 * pixel_index[n, f] among its group's units (4 * rank + offset % 4).  One CTA
 * per (image, group) copies the listed units into shared memory, then writes
 * the group's rows from there: the image is read with coalesced 16-byte
 * copies instead of one scattered load per feature.  image and image_elems
 * must be 16-byte aligned / a multiple of 4.  The plan depends on the patch
 * geometry only; the caller builds it once from pixel_index.                */
typedef struct svit_gather_plan {
  const int32_t* stage_offset; /* sum of the group counts, int32 units, each in [0, image_elems / 4) */
  const int32_t* stage_begin;  /* (groups + 1), stage_begin[0] = 0, non-decreasing */
  const int16_t* local_index;  /* (patches, features) in [0, 4 * group count), 16-byte aligned */
  int64_t groups;              /* ceil(patches / group_patches) */
  int64_t group_patches;
  int64_t max_stage;           /* largest group count; max_stage * 16 bytes <= 227 KB */
} svit_gather_plan;

INTP_API intp_status svit_gather_patches_staged(const float* image, int64_t batch, int64_t image_elems,
                                                const svit_gather_plan* plan, const float* weight,
                                                int64_t patches, int64_t features, void* out, void* stream);

/* Geometry of the post-GEMM step (one response row per patch).
 * resp row layout (bf16): [bases x directions tokenizer scores |
 * for each support s: look_heads x directions Look-bank responses], so Look
 * pose p = s * directions + d of head h sits at column
 * bases*directions + s*look_heads*directions + h*directions + d.            */
typedef struct svit_embed_args {
  int64_t batch, patches;          /* patches per image (N - 1)                    */
  int32_t bases, directions;       /* tokenizer: bases x directions, 2*bases = dim */
  int32_t look_heads, look_poses;  /* look_poses = supports x directions           */
  int32_t slots;                   /* Look slots per head                          */
  const void* resp;   int64_t resp_stride;  /* bf16 (batch*patches, >= columns)    */
  const float* token_null;      /* (bases) null score of each base               */
  const float* direction_coef;  /* (directions, 2) cos / sin of each direction   */
  const float* output_bias;     /* (2*bases)                                     */
  const float* cls;             /* (2*bases) CLS token                           */
  const float* pos_embed;       /* (patches + 1, 2*bases)                        */
  const float* look_null;       /* (look_heads) null score of each Look head     */
  const float* slot_fields;     /* (look_heads, look_poses, slots) Look value of */
                                /* each slot per pose                            */
  float* x;                     /* out: (batch, patches + 1, 2*bases) tokens     */
  float* values;                /* out: (batch, look_heads, patches, slots):     */
                                /* per image and head, the patches' slot values  */
                                /* are contiguous.  May be NULL (see look_pose)  */
  float* look_pose;             /* out (optional): (batch, patches, look_heads,  */
                                /* look_poses) Look pose after the null softmax; */
                                /* with values NULL only x and look_pose are     */
                                /* written (the attention forms the per-slot     */
                                /* values itself, SLA_BIAS_SLOT_FIELDS)          */
} svit_embed_args;

INTP_API intp_status svit_embed_post(const svit_embed_args* args, void* stream);

/* The tokenizer + Look-bank GEMM and svit_embed_post's work in one tcgen05
 * kernel (replaces the reference's rotating-dot responses and the softmaxes
 * that follow them, layers/hex_rotating_harmonic_patch_embed.py:153-242 and
 * layers/square_patch_dense_grid_look.py:339-355): C = patches W^T with fp32
 * accumulators in tensor memory, and from them, without writing C,
 *   x[b, n+1, 2p + c] = sum_d softmax_d,null(C[., 6p + d]) coef[d, c]
 *                       + output_bias[2p + c] + pos_embed[n+1, 2p + c],
 *   x[b, 0] = cls + pos_embed[0],
 *   look_pose[b, n, h, pp] = softmax_pp,null(C[., 6 bases + 12 h + pp]).
 * patches: (batch * args->patches, features) bf16, row stride patches_stride
 * (16-byte aligned rows); weight: (6 bases + 12 look_heads, features) bf16
 * contiguous, the tokenizer rows first, then the Look rows head by head (head
 * h's 12 poses consecutive).  args: directions == 6, look_poses == 12,
 * bases % 24 == 0, look_heads % 12 == 0, values == NULL, x and look_pose set;
 * resp and slot_fields are not used.  features % 8 == 0 (a ragged last
 * 64-wide K slab reads zeros).  x, look_pose, pos_embed, cls and output_bias
 * are 16-byte aligned (INTP_ERR_LAYOUT otherwise).  `status`: the device
 * int32 of the bounded waits (as in sla_forward_args.status).                */
INTP_API intp_status svit_tokenizer_gemm(const svit_embed_args* args, const void* patches, int64_t patches_stride,
                                         int32_t features, const void* weight, int32_t* status, void* stream);

/* For r < rows: x[r] += y[r] (when y is not NULL; y bf16), then
 * h[r] = bf16(LayerNorm(x[r]) * gamma + beta) over `dim` features.
 * Row r of x / y / h starts at r * x_stride / y_stride / h_stride elements.
 * dim % 64 == 0 and dim <= 512.                                             */
INTP_API intp_status svit_add_layernorm(float* x, int64_t x_stride, const void* y, int64_t y_stride,
                                        const float* gamma, const float* beta, float eps, int64_t rows,
                                        int64_t dim, void* h, int64_t h_stride, void* stream);

/* Linear layers of the transformer block on tcgen05 tensor cores with the
 * element-wise work that follows them fused into the epilogue
 * (layers/mini_vit.py:138-170: fc1 -> GELU; proj / fc2 -> residual add ->
 * next pre-norm).  C = A W^T + bias with A (rows, in_features) bf16 (row
 * stride a_stride, 16-byte aligned rows), W (out_features, in_features) bf16
 * contiguous (a torch Linear weight), bias float32; fp32 accumulation.
 * in_features % 64 == 0.  `status` is the device int32 that bounded waits
 * write on failure (as in sla_forward_args.status).
 *
 * svit_linear_gelu: out = bf16(GELU(C)) with the exact error function
 *   (nn.GELU()); out_features % 256 == 0; out row stride % 8 == 0.
 * svit_linear_residual_layernorm: x += C (x float32, updated in place), then
 *   h = bf16(LayerNorm(x) * gamma + beta); dim (= out_features) == 192.
 * svit_linear_bias: out = bf16(C) (the attention's qkv projection,
 *   layers/mini_vit.py:68); out_features % 192 == 0; out row stride % 8 == 0. */
INTP_API intp_status svit_linear_gelu(const void* a, int64_t a_stride, int64_t rows, int32_t in_features,
                                      const void* weight, const float* bias, int32_t out_features, void* out,
                                      int64_t out_stride, int32_t* status, void* stream);
INTP_API intp_status svit_linear_bias(const void* a, int64_t a_stride, int64_t rows, int32_t in_features,
                                      const void* weight, const float* bias, int32_t out_features, void* out,
                                      int64_t out_stride, int32_t* status, void* stream);
INTP_API intp_status svit_linear_residual_layernorm(const void* a, int64_t a_stride, int64_t rows,
                                                    int32_t in_features, const void* weight, const float* bias,
                                                    int32_t dim, float* x, int64_t x_stride, const float* gamma,
                                                    const float* beta, float eps, void* h, int64_t h_stride,
                                                    int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* INTP_SHARE_VIT_H */
