// share_vit_ops.cu - fused steps of the half6d3r SHARE-ViT forward around the
// Look attention (C ABI in include/intp_share_vit.h).
//
// All three kernels are HBM-bound elementwise / gather work: they read their
// inputs once, keep intermediates in registers or shared memory and write
// their outputs once, coalesced.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "../../include/intp_share_vit.h"
#include "sm100_ptx.cuh"

namespace intp {
namespace {

// ------------------------------------------------------------------ gather
// One thread writes 8 consecutive features (16 bytes) of one patch row.
__global__ void __launch_bounds__(256) gather_patches_kernel(const float* __restrict__ image, int64_t image_elems,
                                                             const int32_t* __restrict__ pixel_index,
                                                             const float* __restrict__ weight, int64_t patches,
                                                             int64_t features, int64_t rows,
                                                             uint4* __restrict__ out) {
  const int64_t chunks = features / 8;
  const int64_t total = rows * chunks;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = t / chunks, c = t - row * chunks;
    const int64_t b = row / patches, n = row - b * patches;
    const int4* idx = reinterpret_cast<const int4*>(pixel_index + n * features + c * 8);
    const float4* wt = reinterpret_cast<const float4*>(weight + c * 8);
    const int4 i0 = __ldg(idx), i1 = __ldg(idx + 1);
    const float4 w0 = __ldg(wt), w1 = __ldg(wt + 1);
    const float* img = image + b * image_elems;
    const float v0 = __ldg(img + i0.x) * w0.x, v1 = __ldg(img + i0.y) * w0.y;
    const float v2 = __ldg(img + i0.z) * w0.z, v3 = __ldg(img + i0.w) * w0.w;
    const float v4 = __ldg(img + i1.x) * w1.x, v5 = __ldg(img + i1.y) * w1.y;
    const float v6 = __ldg(img + i1.z) * w1.z, v7 = __ldg(img + i1.w) * w1.w;
    out[t] = make_uint4(pack_bf16x2(v0, v1), pack_bf16x2(v2, v3), pack_bf16x2(v4, v5), pack_bf16x2(v6, v7));
  }
}

// Staged gather: one CTA per (image, patch group).  Phase 1 copies the
// group's distinct 16-byte image units (sorted, so consecutive threads read
// runs of consecutive addresses) into shared memory with cp.async; phase 2
// writes the group's rows, each thread 8 consecutive features (16 bytes),
// from shared memory.  Several CTAs per SM overlap one's copies with
// another's writes: the kernel is latency-bound, so it is compiled for 8 CTAs
// per SM (32 registers) and groups should stay under 28 KB of shared memory.
constexpr int kStagedThreads = 256;

__global__ void __launch_bounds__(kStagedThreads, 8) gather_patches_staged_kernel(
    const float* __restrict__ image, int64_t image_elems, const int32_t* __restrict__ stage_offset,
    const int32_t* __restrict__ stage_begin, const int16_t* __restrict__ local_index,
    const float* __restrict__ weight, int groups, int group_patches, int patches, int features,
    uint4* __restrict__ out) {
  extern __shared__ __align__(16) float staged[];
  const int g = static_cast<int>(blockIdx.x % static_cast<unsigned>(groups));
  const int64_t b = blockIdx.x / static_cast<unsigned>(groups);
  const float4* img = reinterpret_cast<const float4*>(image + b * image_elems);
  const int s0 = __ldg(stage_begin + g), count = __ldg(stage_begin + g + 1) - s0;
  const uint32_t staged_base = smem_u32(staged);
  // Offsets in batches of kStageBatch per thread: the batch's loads are all in
  // flight before its copies are issued (one L2 round trip per batch).
  constexpr int kStageBatch = 8;
  for (int k0 = threadIdx.x; k0 < count; k0 += kStageBatch * kStagedThreads) {
    int off[kStageBatch];
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int k = k0 + u * kStagedThreads;
      off[u] = k < count ? __ldg(stage_offset + s0 + k) : 0;
    }
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int k = k0 + u * kStagedThreads;
      if (k < count)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(staged_base + 16u * k), "l"(img + off[u])
                     : "memory");
    }
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncthreads();

  const int n0 = g * group_patches;
  const int rows = min(group_patches, patches - n0);
  const int chunks = features / 8;
  const uint4* idx = reinterpret_cast<const uint4*>(local_index + static_cast<int64_t>(n0) * features);
  uint4* dst = out + (b * patches + n0) * chunks;
  // Each thread keeps one 8-feature chunk (its weights in registers) for all
  // the group's rows; kRowBatch rows' index words are loaded first.
  constexpr int kRowBatch = 2;
  for (int c = threadIdx.x; c < chunks; c += kStagedThreads) {
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(weight) + 2 * c);
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(weight) + 2 * c + 1);
    for (int r0 = 0; r0 < rows; r0 += kRowBatch) {
      uint4 li[kRowBatch];
#pragma unroll
      for (int u = 0; u < kRowBatch; ++u)
        li[u] = r0 + u < rows ? __ldg(idx + (r0 + u) * chunks + c) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < kRowBatch; ++u) {
        if (r0 + u < rows) {
          const float v0 = staged[li[u].x & 0xffffu] * w0.x, v1 = staged[li[u].x >> 16] * w0.y;
          const float v2 = staged[li[u].y & 0xffffu] * w0.z, v3 = staged[li[u].y >> 16] * w0.w;
          const float v4 = staged[li[u].z & 0xffffu] * w1.x, v5 = staged[li[u].z >> 16] * w1.y;
          const float v6 = staged[li[u].w & 0xffffu] * w1.z, v7 = staged[li[u].w >> 16] * w1.w;
          dst[(r0 + u) * chunks + c] =
              make_uint4(pack_bf16x2(v0, v1), pack_bf16x2(v2, v3), pack_bf16x2(v4, v5), pack_bf16x2(v6, v7));
        }
      }
    }
  }
}

// ------------------------------------------------------------------ post-GEMM
// Geometry fixed at compile time: D directions, LP = supports x D Look poses.
constexpr int kPostTokens = 32;    // patches per CTA
constexpr int kPostThreads = 256;
constexpr int kMaxLookHeads = 64;
constexpr int kMaxSlots = 128;

__device__ __forceinline__ float bf16_at(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }

// Phase 1: one warp per patch - tokenizer moments straight into x, the Look
// pose (null softmax per head) into shared memory.  Phase 2: for each head,
// values[b, h, n, s] = sum_p pose[row, h, p] * fields[h, p, s] with the head's
// fields in shared memory and each thread keeping one slot's column in
// registers while it walks the CTA's patches.
// VALUES: also the per-slot Look values (phase 2); without it the kernel writes
// x and the Look pose only and compiles without the phase-2 registers.
template <int D, int LP, bool VALUES>
__global__ void __launch_bounds__(kPostThreads) embed_post_kernel(const svit_embed_args a) {
  extern __shared__ __align__(16) float smem_post[];
  const int LH = a.look_heads, S = a.slots;
  float* pose_s = smem_post;  // [kPostTokens][LH][LP]
  const int64_t rows = a.batch * a.patches;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kPostTokens;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dim = 2 * a.bases;
  const __nv_bfloat16* resp = static_cast<const __nv_bfloat16*>(a.resp);

  for (int t = warp; t < kPostTokens; t += kPostThreads / 32) {
    const int64_t row = row0 + t;
    if (row >= rows) break;
    const int64_t b = row / a.patches, n = row - b * a.patches;
    const __nv_bfloat16* r = resp + row * a.resp_stride;
    float* xrow = a.x + (b * (a.patches + 1) + n + 1) * dim;
    const float* pos = a.pos_embed + (n + 1) * dim;
    for (int p = lane; p < a.bases; p += 32) {
      // softmax over the directions plus a learned null state; the null's share is dropped
      float sc[D];
      const float null = a.token_null[p];
      float mx = null;
#pragma unroll
      for (int d = 0; d < D; ++d) {
        sc[d] = bf16_at(r, p * D + d);
        mx = fmaxf(mx, sc[d]);
      }
      float sum = __expf(null - mx), tx = 0.f, ty = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) {
        const float e = __expf(sc[d] - mx);
        sum += e;
        tx = fmaf(e, a.direction_coef[2 * d], tx);
        ty = fmaf(e, a.direction_coef[2 * d + 1], ty);
      }
      const float inv = 1.f / sum;
      *reinterpret_cast<float2*>(xrow + 2 * p) =
          make_float2(fmaf(tx, inv, a.output_bias[2 * p] + pos[2 * p]),
                      fmaf(ty, inv, a.output_bias[2 * p + 1] + pos[2 * p + 1]));
    }
    if (n == 0) {  // the CLS row of this image
      float* crow = a.x + b * (a.patches + 1) * dim;
      for (int c = lane; c < dim; c += 32) crow[c] = a.cls[c] + a.pos_embed[c];
    }
    const int64_t look0 = static_cast<int64_t>(a.bases) * D;
    for (int h = lane; h < LH; h += 32) {
      float sc[LP];
      const float null = a.look_null[h];
      float mx = null;
#pragma unroll
      for (int pp = 0; pp < LP; ++pp) {
        sc[pp] = bf16_at(r, look0 + static_cast<int64_t>(pp / D) * LH * D + h * D + pp % D);
        mx = fmaxf(mx, sc[pp]);
      }
      float sum = __expf(null - mx);
#pragma unroll
      for (int pp = 0; pp < LP; ++pp) {
        sc[pp] = __expf(sc[pp] - mx);
        sum += sc[pp];
      }
      const float inv = 1.f / sum;
      if (VALUES) {  // staged for the per-slot products of phase 2
        float* dst = pose_s + (t * LH + h) * LP;
#pragma unroll
        for (int pp = 0; pp < LP; ++pp) dst[pp] = sc[pp] * inv;
      }
      if (a.look_pose != nullptr) {
        float4* g = reinterpret_cast<float4*>(a.look_pose + (row * LH + h) * LP);
#pragma unroll
        for (int c = 0; c < LP / 4; ++c)
          g[c] = make_float4(sc[4 * c] * inv, sc[4 * c + 1] * inv, sc[4 * c + 2] * inv, sc[4 * c + 3] * inv);
      }
    }
  }
  if constexpr (!VALUES) {
    return;
  } else {

  // Phase 2.  Thread -> (head, quad of 4 slots): the quad's 4 x LP fields stay
  // in registers while the thread walks the CTA's patches (48 FMAs per three
  // 16-byte shared loads and one 16-byte store); heads go round by round.
  // out_base[t]: offset of patch t's (head 0, slot 0) value; head h adds h * patches * S.
  __shared__ int64_t out_base[kPostTokens];
  if (threadIdx.x < kPostTokens) {
    const int64_t row = row0 + threadIdx.x;
    const int64_t b = row / a.patches, n = row - b * a.patches;
    out_base[threadIdx.x] = row < rows ? (b * LH * a.patches + n) * S : -1;
  }
  __syncthreads();
  const int quads = S / 4;
  const int heads_per_round = kPostThreads / quads;
  const int64_t head_step = a.patches * S;
  for (int h0 = 0; h0 < LH; h0 += heads_per_round) {
    const int h = h0 + static_cast<int>(threadIdx.x) / quads, q = static_cast<int>(threadIdx.x) % quads;
    if (h >= LH || threadIdx.x >= heads_per_round * quads) continue;
    float4 f[LP];
    const float4* src = reinterpret_cast<const float4*>(a.slot_fields + static_cast<int64_t>(h) * LP * S) + q;
#pragma unroll
    for (int pp = 0; pp < LP; ++pp) f[pp] = __ldg(src + pp * quads);
    const int64_t head_off = h * head_step + 4 * q;
    for (int t = 0; t < kPostTokens; ++t) {
      const int64_t base = out_base[t];
      if (base < 0) break;
      const float4* pose = reinterpret_cast<const float4*>(pose_s + (t * LH + h) * LP);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int c = 0; c < LP / 4; ++c) {
        const float4 p4 = pose[c];
        const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float4 fe = f[4 * c + e];
          v.x = fmaf(pv[e], fe.x, v.x);
          v.y = fmaf(pv[e], fe.y, v.y);
          v.z = fmaf(pv[e], fe.z, v.z);
          v.w = fmaf(pv[e], fe.w, v.w);
        }
      }
      *reinterpret_cast<float4*>(a.values + base + head_off) = v;
    }
  }
  }
}

// ------------------------------------------------------------------ add + LayerNorm
// One warp per row; lane l holds features 64 i + 2 l, 64 i + 2 l + 1 (i < VPT / 2).
template <int VPT>
__global__ void __launch_bounds__(256) add_layernorm_kernel(float* __restrict__ x, int64_t x_stride,
                                                            const __nv_bfloat162* __restrict__ y, int64_t y_stride,
                                                            const float* __restrict__ gamma,
                                                            const float* __restrict__ beta, float eps, int64_t rows,
                                                            __nv_bfloat162* __restrict__ h, int64_t h_stride) {
  constexpr int kPairs = VPT / 2;
  constexpr int kDim = 32 * VPT;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  float2* xr = reinterpret_cast<float2*>(x + row * x_stride);
  float2 v[kPairs];
#pragma unroll
  for (int i = 0; i < kPairs; ++i) v[i] = xr[32 * i + lane];
  if (y != nullptr) {
    const __nv_bfloat162* yr = y + row * (y_stride / 2);
#pragma unroll
    for (int i = 0; i < kPairs; ++i) {
      const float2 u = __bfloat1622float2(yr[32 * i + lane]);
      v[i].x += u.x;
      v[i].y += u.y;
      xr[32 * i + lane] = v[i];
    }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kPairs; ++i) s += v[i].x + v[i].y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s * (1.f / kDim);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kPairs; ++i) {
    const float dx = v[i].x - mean, dy = v[i].y - mean;
    q = fmaf(dx, dx, fmaf(dy, dy, q));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q * (1.f / kDim) + eps);
  const float2* g2 = reinterpret_cast<const float2*>(gamma);
  const float2* b2 = reinterpret_cast<const float2*>(beta);
  __nv_bfloat162* hr = h + row * (h_stride / 2);
#pragma unroll
  for (int i = 0; i < kPairs; ++i) {
    const float2 g = __ldg(g2 + 32 * i + lane), bb = __ldg(b2 + 32 * i + lane);
    hr[32 * i + lane] = __floats2bfloat162_rn(fmaf((v[i].x - mean) * rstd, g.x, bb.x),
                                              fmaf((v[i].y - mean) * rstd, g.y, bb.y));
  }
}

int grid_for(int64_t work, int threads) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sms) * 16;
  return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace
}  // namespace intp

using namespace intp;

extern "C" INTP_API intp_status svit_gather_patches(const float* image, int64_t batch, int64_t image_elems,
                                                    const int32_t* pixel_index, const float* weight, int64_t patches,
                                                    int64_t features, void* out, void* stream) {
  if (batch < 0 || patches < 0 || features < 0 || image_elems < 0) return INTP_ERR_ARGUMENT;
  if (batch == 0 || patches == 0 || features == 0) return INTP_OK;
  if (!image || !pixel_index || !weight || !out) return INTP_ERR_ARGUMENT;
  if (features % 8 || !aligned(pixel_index, 16) || !aligned(weight, 16) || !aligned(out, 16)) return INTP_ERR_LAYOUT;
  const int64_t rows = batch * patches;
  gather_patches_kernel<<<grid_for(rows * (features / 8), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      image, image_elems, pixel_index, weight, patches, features, rows, static_cast<uint4*>(out));
  return cudaGetLastError() == cudaSuccess ? INTP_OK : INTP_ERR_LAUNCH;
}

extern "C" INTP_API intp_status svit_gather_patches_staged(const float* image, int64_t batch, int64_t image_elems,
                                                           const svit_gather_plan* plan, const float* weight,
                                                           int64_t patches, int64_t features, void* out,
                                                           void* stream) {
  if (batch < 0 || patches < 0 || features < 0 || image_elems < 0 || !plan) return INTP_ERR_ARGUMENT;
  if (batch == 0 || patches == 0 || features == 0) return INTP_OK;
  if (!image || !weight || !out || !plan->stage_offset || !plan->stage_begin || !plan->local_index)
    return INTP_ERR_ARGUMENT;
  if (plan->group_patches <= 0 || plan->groups != (patches + plan->group_patches - 1) / plan->group_patches ||
      plan->max_stage < 0)
    return INTP_ERR_ARGUMENT;
  if (features % 8 || image_elems % 4 || !aligned(image, 16) || !aligned(plan->local_index, 16) ||
      !aligned(weight, 16) || !aligned(out, 16))
    return INTP_ERR_LAYOUT;
  constexpr int64_t kMaxShared = 227 * 1024;
  const int64_t smem = plan->max_stage * static_cast<int64_t>(sizeof(float4));
  if (smem > kMaxShared || patches > INT32_MAX / features || batch * plan->groups > INT32_MAX)
    return INTP_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(gather_patches_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return INTP_ERR_LAUNCH;
  gather_patches_staged_kernel<<<static_cast<unsigned>(batch * plan->groups), kStagedThreads, smem,
                                 static_cast<cudaStream_t>(stream)>>>(
      image, image_elems, plan->stage_offset, plan->stage_begin, plan->local_index, weight,
      static_cast<int>(plan->groups), static_cast<int>(plan->group_patches), static_cast<int>(patches),
      static_cast<int>(features), static_cast<uint4*>(out));
  return cudaGetLastError() == cudaSuccess ? INTP_OK : INTP_ERR_LAUNCH;
}

extern "C" INTP_API intp_status svit_embed_post(const svit_embed_args* a, void* stream) {
  if (!a) return INTP_ERR_ARGUMENT;
  if (a->batch < 0 || a->patches < 0) return INTP_ERR_ARGUMENT;
  if (a->batch == 0 || a->patches == 0) return INTP_OK;
  if (a->bases < 1 || a->look_heads < 1 || a->look_heads > kMaxLookHeads || a->slots < 1 || a->slots > kMaxSlots)
    return INTP_ERR_SHAPE;
  // The half6d3r geometry: 6 directions, 2 supports x 6 directions of Look pose.
  if (a->directions != 6 || a->look_poses != 12) return INTP_ERR_UNSUPPORTED;
  static_assert((12 % 4) == 0, "pose rows are read as float4");
  constexpr int D = 6, LP = 12;
  const int64_t columns = static_cast<int64_t>(a->bases) * D + static_cast<int64_t>(LP) * a->look_heads;
  if (a->resp_stride < columns) return INTP_ERR_SHAPE;
  if (!a->resp || !a->token_null || !a->direction_coef || !a->output_bias || !a->cls || !a->pos_embed ||
      !a->look_null || !a->x || (!a->values && !a->look_pose) || (a->values && !a->slot_fields))
    return INTP_ERR_ARGUMENT;
  if (!aligned(a->x, 8)) return INTP_ERR_LAYOUT;
  if (a->values && (a->slots % 4 || !aligned(a->slot_fields, 16) || !aligned(a->values, 16))) return INTP_ERR_LAYOUT;
  if (a->look_pose && !aligned(a->look_pose, 16)) return INTP_ERR_LAYOUT;
  // the pose staging only serves the per-slot products (values); without them
  // the kernel needs no shared memory and more CTAs fit on an SM
  const size_t smem = a->values ? static_cast<size_t>(kPostTokens) * a->look_heads * LP * sizeof(float) : 0;
  if (smem > 200 * 1024) return INTP_ERR_SHAPE;
  auto kernel = a->values ? embed_post_kernel<D, LP, true> : embed_post_kernel<D, LP, false>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return INTP_ERR_LAUNCH;
  const int64_t blocks = (a->batch * a->patches + kPostTokens - 1) / kPostTokens;
  kernel<<<static_cast<unsigned>(blocks), kPostThreads, smem, static_cast<cudaStream_t>(stream)>>>(*a);
  return cudaGetLastError() == cudaSuccess ? INTP_OK : INTP_ERR_LAUNCH;
}

extern "C" INTP_API intp_status svit_add_layernorm(float* x, int64_t x_stride, const void* y, int64_t y_stride,
                                                   const float* gamma, const float* beta, float eps, int64_t rows,
                                                   int64_t dim, void* h, int64_t h_stride, void* stream) {
  if (rows < 0) return INTP_ERR_ARGUMENT;
  if (rows == 0) return INTP_OK;
  if (!x || !gamma || !beta || !h) return INTP_ERR_ARGUMENT;
  if (dim < 64 || dim > 512 || dim % 64) return INTP_ERR_SHAPE;
  if (x_stride < dim || h_stride < dim || (y && y_stride < dim)) return INTP_ERR_LAYOUT;
  if (x_stride % 2 || h_stride % 2 || (y && y_stride % 2) || !aligned(x, 8) || !aligned(h, 4) ||
      (y && !aligned(y, 4)) || !aligned(gamma, 8) || !aligned(beta, 8))
    return INTP_ERR_LAYOUT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  const auto* yy = static_cast<const __nv_bfloat162*>(y);
  auto* hh = static_cast<__nv_bfloat162*>(h);
  switch (dim / 32) {
    case 2: add_layernorm_kernel<2><<<blocks, 256, 0, s>>>(x, x_stride, yy, y_stride, gamma, beta, eps, rows, hh, h_stride); break;
    case 4: add_layernorm_kernel<4><<<blocks, 256, 0, s>>>(x, x_stride, yy, y_stride, gamma, beta, eps, rows, hh, h_stride); break;
    case 6: add_layernorm_kernel<6><<<blocks, 256, 0, s>>>(x, x_stride, yy, y_stride, gamma, beta, eps, rows, hh, h_stride); break;
    case 8: add_layernorm_kernel<8><<<blocks, 256, 0, s>>>(x, x_stride, yy, y_stride, gamma, beta, eps, rows, hh, h_stride); break;
    case 10: add_layernorm_kernel<10><<<blocks, 256, 0, s>>>(x, x_stride, yy, y_stride, gamma, beta, eps, rows, hh, h_stride); break;
    case 12: add_layernorm_kernel<12><<<blocks, 256, 0, s>>>(x, x_stride, yy, y_stride, gamma, beta, eps, rows, hh, h_stride); break;
    case 14: add_layernorm_kernel<14><<<blocks, 256, 0, s>>>(x, x_stride, yy, y_stride, gamma, beta, eps, rows, hh, h_stride); break;
    case 16: add_layernorm_kernel<16><<<blocks, 256, 0, s>>>(x, x_stride, yy, y_stride, gamma, beta, eps, rows, hh, h_stride); break;
    default: return INTP_ERR_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? INTP_OK : INTP_ERR_LAUNCH;
}
