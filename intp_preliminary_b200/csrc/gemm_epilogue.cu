// gemm_epilogue.cu - tcgen05 GEMM with the transformer block's element-wise
// work fused into its epilogue (C ABI in include/intp_share_vit.h).
//
//   C[M, N] = A[M, K] W[N, K]^T + bias     (bf16 operands, fp32 accumulation in TMEM)
//   GELU epilogue:      out = bf16(GELU_erf(C))                       (MLP fc1)
//   bias epilogue:      out = bf16(C)                                  (attention qkv)
//   residual + LN:      x += C (fp32);  h = bf16(LayerNorm(x))         (attention proj, MLP fc2)
//   tokenizer:          the patch tokenizer's and the Look bank's null softmaxes straight
//                       from the fp32 accumulators (no response matrix in memory):
//                       tokens x (harmonic moments + bias + position, CLS row) and the
//                       Look pose, layers/hex_rotating_harmonic_patch_embed.py:153-242 and
//                       layers/square_patch_dense_grid_look.py:339-355
// so the MLP's 768-wide activation is written once (by fc1, already
// activated) and the residual stream is read and written once per sub-block,
// with no separate GELU or add + LayerNorm pass (layers/mini_vit.py:138-170).
//
// CTA (one per SM, persistent over 128-row x NT-column tiles): warp 0 issues
// TMA loads of 64-wide K slabs of A and W into a STAGES-deep ring (128-byte
// swizzle); warp 1 issues tcgen05.mma (M = 128, N = NT, K = 16 per
// instruction) into one of two TMEM accumulators; two groups of four
// epilogue warps (2-5, 6-9: warp w reads TMEM lanes 32 (w % 4) .. + 31) take
// alternate tiles and run the epilogue from TMEM, one row per thread, while
// the next tile accumulates in the other buffer.  The tokenizer instead takes
// 256-row tiles as two 128-row accumulators that share each weight slab
// (half the weight's trips through shared memory per row); its 2 x 144 TMEM
// columns leave no room for a second buffer, so both epilogue groups drain
// one tile together, each its own 128 rows, and hand the accumulator back as
// soon as it sits in registers.  Every wait is bounded (sm100_ptx.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>
#include "../../include/intp_share_vit.h"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace intp {
namespace {

constexpr int kGBM = 128;                          // rows per tile
constexpr int kGBK = 64;                           // K per slab: 128 bytes of bf16 = one swizzle atom
constexpr uint32_t kASlab = kGBM * kGBK * 2;       // 16 KB
// Warps: 0 TMA, 1 MMA, then groups of four epilogue warps.  Two groups per
// accumulator buffer for GELU (each takes half of the tile's columns), one for
// LayerNorm (a row's statistics stay inside one thread).
template <int EPI>
__host__ __device__ constexpr int epi_groups_per_tile() { return EPI == 1 || EPI == 3 ? 1 : 2; }
template <int EPI>
__host__ __device__ constexpr int gemm_threads() { return 64 + 2 * epi_groups_per_tile<EPI>() * 128; }
constexpr int kEpiGelu = 0, kEpiResidualLN = 1, kEpiBias = 2, kEpiTokenizer = 3;
// 128-row sub-tiles per tile (sharing the weight slab) and TMEM accumulator buffers.
template <int EPI>
__host__ __device__ constexpr int m_subtiles() { return EPI == 3 ? 2 : 1; }
template <int EPI>
__host__ __device__ constexpr int acc_buffers() { return EPI == 3 ? 1 : 2; }
// Per epilogue warp, in 32-bit words: GELU two 32 x 32 bf16 blocks; LN two 32 x 32 fp32 residual chunks;
// tokenizer 32 rows x 52 fp32.
template <int EPI>
__host__ __device__ constexpr int stage_words() { return EPI == 3 ? 32 * 52 : (EPI == 1 ? 2048 : 1024); }
constexpr int kMaxGeluN = 4096;         // GELU bias columns kept in shared memory
constexpr uint32_t kBarrierBytes = 256;  // room reserved for the barrier block

struct GemmArgs {
  int64_t M;
  int32_t N, K;
  int32_t n_tiles_n;   // N / NT
  int64_t tiles;       // ceil(M / (128 * row sub-tiles)) * n_tiles_n
  const float* bias;   // (N)
  __nv_bfloat16* out;  // GELU: (M, N) bf16, row stride out_stride
  int64_t out_stride;
  float* x;            // LN: residual (M, N) fp32, row stride x_stride, updated in place
  int64_t x_stride;
  const float* gamma;
  const float* beta;
  float eps;
  __nv_bfloat16* h;    // LN: output (M, N) bf16, row stride h_stride
  int64_t h_stride;
  int32_t* status;
  // tokenizer epilogue (EPI 3): rows are (image, patch) pairs; tiles 0 .. tok_tiles-1
  // cover the tokenizer's bases, the rest the Look bank's heads
  int32_t patches;             // patches per image
  int32_t tok_tiles;           // N-tiles of tokenizer columns
  const float* token_null;     // (bases)
  const float* direction_coef; // (6, 2)
  const float* output_bias;    // (2 bases)
  const float* cls;            // (2 bases)
  const float* pos_embed;      // (patches + 1, 2 bases)
  const float* look_null;      // (look heads)
  float* look_pose;            // (rows, look heads, 12)
  int32_t look_heads;
};

template <int STAGES>
struct GemmBarriers {
  uint64_t full[STAGES], empty[STAGES];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t drain;
  uint64_t params;  // the epilogue parameters have landed in shared memory
  uint32_t tmem_base;
  int32_t abort;
};

// GELU with the error function (nn.GELU(), not its tanh approximation), for
// two columns at once on the packed fp32 pipe.
//
// erf by Abramowitz & Stegun, Handbook of Mathematical Functions, formula
// 7.1.28: for z >= 0, erf(z) = 1 - (1 + a1 z + ... + a6 z^6)^-16, |error| <=
// 3e-7 (about 2e-6 in fp32 arithmetic) - far below the bf16 resolution of the
// output.  With z = |v| / sqrt(2) and q = (1 + ... )^-16 = erfc(z):
//   GELU(v) = v (1 + erf(v / sqrt 2)) / 2 = max(v, 0) - |v| q / 2
// for either sign of v.  One reciprocal (MUFU) per column; the sqrt(2) is
// folded into the coefficients (c_k = a_k 2^(-k/2)).  NaN propagates.
constexpr float kErfC1 = 0.0705230784f * 0.70710678118654752f;
constexpr float kErfC2 = 0.0422820123f * 0.5f;
constexpr float kErfC3 = 0.0092705272f * 0.35355339059327376f;
constexpr float kErfC4 = 0.0001520143f * 0.25f;
constexpr float kErfC5 = 0.0002765672f * 0.17677669529663688f;
constexpr float kErfC6 = 0.0000430638f * 0.125f;

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float2 splat2(float s) { return make_float2(s, s); }

__device__ __forceinline__ uint32_t gelu_bf16x2(float2 v) {
  const float2 av = make_float2(fabsf(v.x), fabsf(v.y));
  float2 p = fma2(splat2(kErfC6), av, splat2(kErfC5));
  p = fma2(p, av, splat2(kErfC4));
  p = fma2(p, av, splat2(kErfC3));
  p = fma2(p, av, splat2(kErfC2));
  p = fma2(p, av, splat2(kErfC1));
  p = fma2(p, av, splat2(1.f));
  float2 q = make_float2(rcp_approx(p.x), rcp_approx(p.y));
  q = mul2(q, q);
  q = mul2(q, q);
  q = mul2(q, q);
  q = mul2(q, q);
  const float2 out = fma2(mul2(av, q), splat2(-0.5f), make_float2(fmaxf(v.x, 0.f), fmaxf(v.y, 0.f)));
  return pack_bf16x2(out.x, out.y);
}

// Per-warp bf16 staging of a 32-row x 32-column block: row r holds 64 bytes
// (four 16-byte chunks), chunk q stored at position q ^ ((r >> 1) & 3), so
// that the row-per-thread 128-bit writes and the 8-rows-per-instruction
// 128-bit reads are both free of bank conflicts.
__device__ __forceinline__ void stage_row_bf16(uint32_t* stage, int row, const uint32_t (&w)[16]) {
  const int sw = (row >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(stage + row * 16 + 4 * (q ^ sw)) = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
}

// Writes the staged block to dst rows [row0, row0 + 32) x 32 columns (bf16),
// 16 bytes per lane, 8 full 64-byte row segments per instruction.
__device__ __forceinline__ void store_staged_bf16(const uint32_t* stage, int lane, __nv_bfloat16* dst, int64_t stride,
                                                  int64_t row0, int64_t rows) {
  const int q = lane & 3;
  uint4 val[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int rr = 8 * j + (lane >> 2);
    val[j] = *reinterpret_cast<const uint4*>(stage + rr * 16 + 4 * (q ^ ((rr >> 1) & 3)));
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t m = row0 + 8 * j + (lane >> 2);
    if (m < rows) *reinterpret_cast<uint4*>(dst + m * stride + 8 * q) = val[j];
  }
}

__device__ __forceinline__ float2 f2(uint32_t lo, uint32_t hi) { return make_float2(__uint_as_float(lo), __uint_as_float(hi)); }

// Hands the accumulator buffer back to the MMA warp once this warp's TMEM reads are complete.
__device__ __forceinline__ void release_acc(uint64_t* acc_empty, int lane) {
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(acc_empty);
}

// fp32 staging of a 32-row x 32-column block (per warp): row r holds eight
// 16-byte chunks, chunk q stored at position q ^ (r & 7).  Row-per-thread
// 128-bit accesses and column-per-lane 32-bit accesses are both conflict free.
__device__ __forceinline__ int fstage_index(int row, int col) {
  return row * 32 + 4 * ((col >> 2) ^ (row & 7)) + (col & 3);
}

// GELU epilogue of one warp: 32 rows x NT columns from TMEM (row = lane),
// 32 columns per step; the next step's TMEM load is in flight while this one
// computes, and the accumulator is released as soon as the last load landed.
template <int NT, bool GELU>
__device__ __forceinline__ void epilogue_gelu(uint32_t acc, const float* sbias, uint32_t* stage, int lane,
                                              __nv_bfloat16* out, int64_t out_stride, int64_t wrow0, int64_t rows,
                                              uint64_t* acc_empty) {
  constexpr int kSteps = NT / 32;
  uint32_t lo[2][16], hi[2][16];
  tmem_ld16(acc, lo[0]);
  tmem_ld16(acc + 16, hi[0]);
  tmem_wait_ld();
  reg_fence16(lo[0]);
  reg_fence16(hi[0]);
#pragma unroll
  for (int s = 0; s < kSteps; ++s) {
    const int b = s & 1;
    if (s + 1 < kSteps) {
      tmem_ld16(acc + 32 * (s + 1), lo[b ^ 1]);
      tmem_ld16(acc + 32 * (s + 1) + 16, hi[b ^ 1]);
    } else {
      release_acc(acc_empty, lane);
    }
    uint32_t w[16];
#pragma unroll
    for (int q = 0; q < 8; ++q) {  // columns 32 s + 4 q .. + 3
      const float4 bb = reinterpret_cast<const float4*>(sbias + 32 * s)[q];
      const uint32_t* r = q < 4 ? lo[b] : hi[b];
      const int j = 4 * (q & 3);
      const float2 v0 = add2(f2(r[j], r[j + 1]), make_float2(bb.x, bb.y));
      const float2 v1 = add2(f2(r[j + 2], r[j + 3]), make_float2(bb.z, bb.w));
      w[2 * q] = GELU ? gelu_bf16x2(v0) : pack_bf16x2(v0.x, v0.y);
      w[2 * q + 1] = GELU ? gelu_bf16x2(v1) : pack_bf16x2(v1.x, v1.y);
    }
    uint32_t* sb = stage + 512 * b;
    stage_row_bf16(sb, lane, w);
    __syncwarp();
    store_staged_bf16(sb, lane, out + 32 * s, out_stride, wrow0, rows);
    if (s + 1 < kSteps) {
      tmem_wait_ld();
      reg_fence16(lo[b ^ 1]);
      reg_fence16(hi[b ^ 1]);
    }
  }
  __syncwarp();
}

// Residual chunk copy: rows [row0, row0 + 32) x 32 fp32 columns of x into a
// per-warp buffer in the fstage layout, 16 bytes per lane per instruction (8
// lanes per 128-byte row segment), asynchronously (cp.async, no registers).
// Rows past the matrix are zero-filled without reading.
__device__ __forceinline__ void copy_x_chunk(float* buf, const float* x, int64_t x_stride, int64_t row0, int64_t rows,
                                             int col0, int lane) {
  const int q = lane & 7;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int r = 4 * j + (lane >> 3);
    const bool in = row0 + r < rows;
    const float* src = in ? x + (row0 + r) * x_stride + col0 + 4 * q : x;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(buf + fstage_index(r, 4 * q))),
                 "l"(src), "r"(in ? 16 : 0)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Residual + LayerNorm epilogue of one warp (32 rows = lanes, NT columns):
//   pass 1, 32 columns per step: v = C + bias + x (row per thread, x from the
//     step's buffer); v written over x in the buffer and from there back to x
//     in global memory (coalesced); v into TMEM; the step's row mean and sum
//     of squared deviations merged into the running ones (Chan, Golub &
//     LeVeque's pairwise update), so no separate variance pass;
//   pass 2: h = bf16((v - mean) rstd gamma + beta).
// The residual chunk of step s + 1 is copied while step s works; the caller
// started the copy of step 0 into xbuf[0] before the accumulator was ready.
template <int NT>
__device__ __forceinline__ void epilogue_residual_ln(uint32_t acc, const float* sparams, float* xbuf, int lane,
                                                     float* x, int64_t x_stride, float eps, __nv_bfloat16* h,
                                                     int64_t h_stride, int64_t wrow0, int64_t rows,
                                                     uint64_t* acc_empty) {
  constexpr int kSteps = NT / 32;
  const float* sbias = sparams;
  const float* sgamma = sparams + NT;
  const float* sbeta = sparams + 2 * NT;
  float mean = 0.f, m2 = 0.f;
#pragma unroll 1
  for (int s = 0; s < kSteps; ++s) {
    const int c = 32 * s;
    float* buf = xbuf + 1024 * (s & 1);
    if (s + 1 < kSteps) copy_x_chunk(xbuf + 1024 * ((s + 1) & 1), x, x_stride, wrow0, rows, c + 32, lane);
    uint32_t lo[16], hi[16];
    tmem_ld16(acc + c, lo);
    tmem_ld16(acc + c + 16, hi);
    if (s + 1 < kSteps)
      cp_async_wait<1>();
    else
      cp_async_wait<0>();
    __syncwarp();
    tmem_wait_ld();
    reg_fence16(lo);
    reg_fence16(hi);
    // all loads of the row first, then the stores (the cells are written in place)
    float4 xv[8], bb[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      xv[q] = *reinterpret_cast<const float4*>(buf + fstage_index(lane, 4 * q));
      bb[q] = reinterpret_cast<const float4*>(sbias + c)[q];
    }
    float2 p[16];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t* r = q < 4 ? lo : hi;
      const int j = 4 * (q & 3);
      p[2 * q] = add2(add2(f2(r[j], r[j + 1]), make_float2(bb[q].x, bb[q].y)), make_float2(xv[q].x, xv[q].y));
      p[2 * q + 1] = add2(add2(f2(r[j + 2], r[j + 3]), make_float2(bb[q].z, bb[q].w)), make_float2(xv[q].z, xv[q].w));
    }
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<float4*>(buf + fstage_index(lane, 4 * q)) =
          make_float4(p[2 * q].x, p[2 * q].y, p[2 * q + 1].x, p[2 * q + 1].y);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      lo[2 * k] = __float_as_uint(p[k].x);
      lo[2 * k + 1] = __float_as_uint(p[k].y);
      hi[2 * k] = __float_as_uint(p[8 + k].x);
      hi[2 * k + 1] = __float_as_uint(p[8 + k].y);
    }
    tmem_st16(acc + c, lo);
    tmem_st16(acc + c + 16, hi);
    __syncwarp();
    {  // v back to the residual stream: 4 rows x 128 bytes per instruction
      const int q = lane & 7;
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = *reinterpret_cast<const float4*>(buf + fstage_index(4 * j + (lane >> 3), 4 * q));
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = 4 * j + (lane >> 3);
        if (wrow0 + r < rows) *reinterpret_cast<float4*>(x + (wrow0 + r) * x_stride + c + 4 * q) = v[j];
      }
    }
    // step statistics: pairwise sums, then the squared deviations about the step mean
    float2 t4[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) t4[k] = add2(add2(p[4 * k], p[4 * k + 1]), add2(p[4 * k + 2], p[4 * k + 3]));
    const float2 t2 = add2(add2(t4[0], t4[1]), add2(t4[2], t4[3]));
    const float mb = (t2.x + t2.y) * (1.f / 32.f);
    float2 d4[4] = {splat2(0.f), splat2(0.f), splat2(0.f), splat2(0.f)};
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float2 d = add2(p[k], splat2(-mb));
      d4[k & 3] = fma2(d, d, d4[k & 3]);
    }
    const float2 dd = add2(add2(d4[0], d4[1]), add2(d4[2], d4[3]));
    const float m2b = dd.x + dd.y;
    if (s == 0) {
      mean = mb;
      m2 = m2b;
    } else {
      // weight of the merge: 32 new values on top of 32 s (approximate reciprocal:
      // statistics only)
      const float kNew = __fdividef(1.f, static_cast<float>(s + 1));
      const float delta = mb - mean;
      mean = fmaf(delta, kNew, mean);
      m2 += fmaf(delta * delta, 32.f * s * kNew, m2b);
    }
    __syncwarp();
  }
  tmem_wait_st();
  const float rstd = rsqrtf(m2 * (1.f / NT) + eps);
  const float2 neg_mean = splat2(-mean), rstd2 = splat2(rstd);
  uint32_t* stage = reinterpret_cast<uint32_t*>(xbuf);
  uint32_t lo[2][16], hi[2][16];
  tmem_ld16(acc, lo[0]);
  tmem_ld16(acc + 16, hi[0]);
  tmem_wait_ld();
  reg_fence16(lo[0]);
  reg_fence16(hi[0]);
#pragma unroll
  for (int s = 0; s < kSteps; ++s) {
    const int c = 32 * s, b = s & 1;
    if (s + 1 < kSteps) {
      tmem_ld16(acc + c + 32, lo[b ^ 1]);
      tmem_ld16(acc + c + 48, hi[b ^ 1]);
    } else {
      release_acc(acc_empty, lane);
    }
    uint32_t w[16];
#pragma unroll
    for (int q = 0; q < 8; ++q) {  // columns c + 4 q .. + 3
      const float4 ga = reinterpret_cast<const float4*>(sgamma + c)[q];
      const float4 be = reinterpret_cast<const float4*>(sbeta + c)[q];
      const uint32_t* r = q < 4 ? lo[b] : hi[b];
      const int j = 4 * (q & 3);
      const float2 d0 = mul2(add2(f2(r[j], r[j + 1]), neg_mean), rstd2);
      const float2 d1 = mul2(add2(f2(r[j + 2], r[j + 3]), neg_mean), rstd2);
      const float2 o0 = fma2(d0, make_float2(ga.x, ga.y), make_float2(be.x, be.y));
      const float2 o1 = fma2(d1, make_float2(ga.z, ga.w), make_float2(be.z, be.w));
      w[2 * q] = pack_bf16x2(o0.x, o0.y);
      w[2 * q + 1] = pack_bf16x2(o1.x, o1.y);
    }
    uint32_t* sb = stage + 512 * b;
    stage_row_bf16(sb, lane, w);
    __syncwarp();
    store_staged_bf16(sb, lane, h + c, h_stride, wrow0, rows);
    if (s + 1 < kSteps) {
      tmem_wait_ld();
      reg_fence16(lo[b ^ 1]);
      reg_fence16(hi[b ^ 1]);
    }
  }
  __syncwarp();
}

// Tokenizer epilogue of one warp (32 rows = lanes) on a 144-column tile: 24
// tokenizer bases x 6 directions, or 12 Look heads x 12 poses (the weight's
// Look rows are ordered head by head).  The thread's whole 144-column row
// is loaded into registers and the accumulator released before any math, so
// that the next tile's MMAs (single TMEM buffer) wait only for the loads.
//   base p: s_d = C[6p + d], null n_p: e_d = exp(s_d - m), m = max(n_p, s),
//     x[2p + c] = sum_d e_d coef[d, c] / (exp(n_p - m) + sum_d e_d) + bias + pos
//   head h: pose[pp] = exp(s_pp - m) / (exp(n_h - m) + sum exp(s - m))
// (the null state's share is dropped, as in the reference).
// A tile's outputs are 48 floats per row (a token tile's 24 bases x 2; a
// Look step of 4 heads x 12), contiguous in x / the Look pose, with rows far
// apart.  They pass through a per-warp staging block (32 rows x 52 floats:
// the padding makes the row-per-thread float4 accesses conflict free), so
// that global memory sees whole 16-byte chunks of consecutive rows, 12 per
// row, from all 32 lanes at once - not 32 scattered rows per instruction.
// The position-embedding rows of a token tile come in the same way.
constexpr int kTokDirs = 6, kLookPoses = 12, kTokTileN = 144;
constexpr int kTokChunk = 48, kTokStageStride = 52;  // floats per row: used, allocated

// Copies the warp's 32 staged rows to / from global memory: row r at
// base + offset of lane r (each lane passes its own row's offset), 48 floats
// each, as 12 float4 per row spread over the lanes; rows with keep == false
// (of lane r) are skipped.
template <bool kToGlobal>
__device__ __forceinline__ void tok_rows_copy(float* stage, float* base, int64_t offset, bool keep, int lane) {
#pragma unroll
  for (int j = 0; j < 32 * (kTokChunk / 4) / 32; ++j) {
    const int idx = lane + 32 * j, rr = idx / (kTokChunk / 4), ch = idx - rr * (kTokChunk / 4);
    const int64_t off = __shfl_sync(0xffffffffu, offset, rr);
    const bool k = __shfl_sync(0xffffffffu, keep, rr);
    float4* sm = reinterpret_cast<float4*>(stage + rr * kTokStageStride) + ch;
    if (kToGlobal) {
      if (k) reinterpret_cast<float4*>(base + off)[ch] = *sm;
    } else {
      *sm = __ldg(reinterpret_cast<const float4*>(base + off) + ch);
    }
  }
}

// A token tile's position-embedding rows into the staging block, fetched
// while the tile still accumulates (the accumulator registers are not live yet).
__device__ __forceinline__ void tokenizer_stage_pos(int64_t tile_n, int64_t m, const GemmArgs& g, int lane,
                                                    float* stage) {
  if (tile_n >= g.tok_tiles) return;
  const int64_t n = m < g.M ? m % g.patches : 0;
  const int dim = 2 * static_cast<int>(g.tok_tiles) * (kTokTileN / kTokDirs);
  tok_rows_copy<false>(stage, const_cast<float*>(g.pos_embed), (n + 1) * dim + tile_n * 2 * (kTokTileN / kTokDirs),
                       true, lane);
  __syncwarp();
}

__device__ __forceinline__ void epilogue_tokenizer(uint32_t acc, int64_t tile_n, int64_t m, const GemmArgs& g,
                                                   int lane, float* stage, uint64_t* acc_empty) {
  uint32_t r[kTokTileN / 16][16];
#pragma unroll
  for (int c = 0; c < kTokTileN / 16; ++c) tmem_ld16(acc + 16 * c, r[c]);
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < kTokTileN / 16; ++c) reg_fence16(r[c]);
  release_acc(acc_empty, lane);
  const bool valid = m < g.M;
  const int64_t img = valid ? m / g.patches : 0, n = valid ? m - img * g.patches : 0;
  const int dim = 2 * static_cast<int>(g.tok_tiles) * (kTokTileN / kTokDirs);  // 2 * bases
  float* srow = stage + lane * kTokStageStride;
  if (tile_n < g.tok_tiles) {
    const int p0 = static_cast<int>(tile_n) * (kTokTileN / kTokDirs);  // first base of the tile
    const int c0 = 2 * p0;                                             // its first x column
    // the staging block holds this tile's position rows (tokenizer_stage_pos)
#pragma unroll
    for (int i2 = 0; i2 < kTokTileN / kTokDirs; i2 += 2) {
      float out[4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = i2 + u, p = p0 + i;
        float s[kTokDirs];
#pragma unroll
        for (int d = 0; d < kTokDirs; ++d) s[d] = __uint_as_float(r[(kTokDirs * i + d) >> 4][(kTokDirs * i + d) & 15]);
        const float nul = __ldg(g.token_null + p);
        float mx = nul;
#pragma unroll
        for (int d = 0; d < kTokDirs; ++d) mx = fmaxf(mx, s[d]);
        float sum = __expf(nul - mx), tx = 0.f, ty = 0.f;
#pragma unroll
        for (int d = 0; d < kTokDirs; ++d) {
          const float e = __expf(s[d] - mx);
          sum += e;
          tx = fmaf(e, __ldg(g.direction_coef + 2 * d), tx);
          ty = fmaf(e, __ldg(g.direction_coef + 2 * d + 1), ty);
        }
        const float inv = 1.f / sum;
        out[2 * u] = tx * inv;
        out[2 * u + 1] = ty * inv;
      }
      float4* cell = reinterpret_cast<float4*>(srow + 2 * i2);
      const float4 pos = *cell, bias = __ldg(reinterpret_cast<const float4*>(g.output_bias + c0 + 2 * i2));
      *cell = make_float4(out[0] + (bias.x + pos.x), out[1] + (bias.y + pos.y), out[2] + (bias.z + pos.z),
                          out[3] + (bias.w + pos.w));
    }
    __syncwarp();
    tok_rows_copy<true>(stage, g.x, (img * (g.patches + 1) + n + 1) * dim + c0, valid, lane);
    if (valid && n == 0) {  // this image's CLS row, the same 48 columns
      float4* crow = reinterpret_cast<float4*>(g.x + img * (g.patches + 1) * dim + c0);
#pragma unroll 4
      for (int c = 0; c < kTokChunk / 4; ++c) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(g.cls + c0) + c);
        const float4 b = __ldg(reinterpret_cast<const float4*>(g.pos_embed + c0) + c);
        crow[c] = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
      }
    }
    __syncwarp();
  } else {
    const int h0 = static_cast<int>(tile_n - g.tok_tiles) * (kTokTileN / kLookPoses);
#pragma unroll
    for (int st = 0; st < kTokTileN / kTokChunk; ++st) {
#pragma unroll
      for (int i = 0; i < kTokChunk / kLookPoses; ++i) {
        const int col = kTokChunk * st + kLookPoses * i, hh = h0 + col / kLookPoses;
        float e[kLookPoses];
#pragma unroll
        for (int pp = 0; pp < kLookPoses; ++pp) e[pp] = __uint_as_float(r[(col + pp) >> 4][(col + pp) & 15]);
        const float nul = __ldg(g.look_null + hh);
        float mx = nul;
#pragma unroll
        for (int pp = 0; pp < kLookPoses; ++pp) mx = fmaxf(mx, e[pp]);
        float sum = __expf(nul - mx);
#pragma unroll
        for (int pp = 0; pp < kLookPoses; ++pp) {
          e[pp] = __expf(e[pp] - mx);
          sum += e[pp];
        }
        const float inv = 1.f / sum;
        float4* cell = reinterpret_cast<float4*>(srow + kLookPoses * i);
#pragma unroll
        for (int c = 0; c < kLookPoses / 4; ++c)
          cell[c] = make_float4(e[4 * c] * inv, e[4 * c + 1] * inv, e[4 * c + 2] * inv, e[4 * c + 3] * inv);
      }
      __syncwarp();
      tok_rows_copy<true>(stage, g.look_pose, (m * g.look_heads + h0 + st * (kTokChunk / kLookPoses)) * kLookPoses,
                          valid, lane);
      __syncwarp();
    }
  }
}

template <int NT, int STAGES, int EPI>
__global__ void __launch_bounds__(gemm_threads<EPI>(), 1)
gemm_epilogue_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const GemmArgs g) {
  constexpr int kMSub = m_subtiles<EPI>(), kBufs = acc_buffers<EPI>();
  constexpr int64_t kTileM = kMSub * kGBM;
  constexpr uint32_t kBSlab = NT * kGBK * 2;
  constexpr uint32_t kStage = kMSub * kASlab + kBSlab;  // A sub-tiles, then the weight slab
  constexpr uint32_t kTmemCols = kBufs * kMSub * NT <= 256 ? 256 : 512;
  static_assert(kBufs * kMSub * NT <= 512, "TMEM columns");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  GemmBarriers<STAGES>* bars = reinterpret_cast<GemmBarriers<STAGES>*>(smem + STAGES * kStage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int32_t* abort_flag = &bars->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 4 * epi_groups_per_tile<EPI>() * kMSub);
    }
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->params, 1);
    bars->abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const int n_slabs = (g.K + kGBK - 1) / kGBK;  // a ragged last slab reads zeros past K

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      uint32_t loads = 0, stage = 0, phase = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
        const int32_t m0 = static_cast<int32_t>((t / g.n_tiles_n) * kTileM);
        const int32_t n0 = static_cast<int32_t>((t % g.n_tiles_n) * NT);
        // a second row sub-tile wholly past M is neither loaded nor multiplied
        const bool sub1 = kMSub == 2 && m0 + kGBM < g.M;
        const uint32_t bytes = kStage - (kMSub == 2 && !sub1 ? kASlab : 0u);
        for (int ks = 0; ks < n_slabs; ++ks) {
          if (loads >= STAGES &&
              !mbar_wait(&bars->empty[stage], phase ^ 1u, abort_flag, g.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + stage * kStage;
          mbar_arrive_expect_tx(&bars->full[stage], bytes);
          tma_load_2d(dst, &tm_a, &bars->full[stage], ks * kGBK, m0);
          if (sub1) tma_load_2d(dst + kASlab, &tm_a, &bars->full[stage], ks * kGBK, m0 + kGBM);
          tma_load_2d(dst + kMSub * kASlab, &tm_b, &bars->full[stage], ks * kGBK, n0);
          ++loads;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: stage s received (loads - s + STAGES - 1) / STAGES loads.
      volatile int32_t no_abort = 0;
      for (uint32_t s = 0; s < STAGES; ++s) {
        const uint32_t cnt = loads > s ? (loads - s + STAGES - 1) / STAGES : 0;
        if (cnt > 0) mbar_wait(&bars->full[s], (cnt - 1) & 1, &no_abort, g.status, kDevTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(true, false, kGBM, NT);
      const uint64_t a_desc = smem_desc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t b_desc = smem_desc_sw128(smem_u32(smem + kMSub * kASlab), 16, 1024);
      uint32_t stage = 0, phase = 0, lt = 0;
      bool ok = true, issued = false;
      for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x, ++lt) {
        const uint32_t buf = lt % kBufs;
        if (lt >= kBufs &&
            !mbar_wait(&bars->acc_empty[buf], ((lt - kBufs) / kBufs) & 1, abort_flag, g.status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        const bool sub1 = kMSub == 2 && (t / g.n_tiles_n) * kTileM + kGBM < g.M;
        const uint32_t d_tmem = tmem + buf * kMSub * NT;
        tc_fence_after();
        for (int ks = 0; ks < n_slabs; ++ks) {
          if (!mbar_wait(&bars->full[stage], phase, abort_flag, g.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kGBK / 16; ++kk) {
            const uint64_t b_k = b_desc + ((stage * kStage + kk * 32) >> 4);
            mma_ss(d_tmem, a_desc + ((stage * kStage + kk * 32) >> 4), b_k, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
            if (sub1)
              mma_ss(d_tmem + NT, a_desc + ((stage * kStage + kASlab + kk * 32) >> 4), b_k, idesc,
                     (ks > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&bars->empty[stage]);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&bars->acc_full[buf]);
      }
      if (issued) {
        mma_commit(&bars->drain);
        volatile int32_t no_abort = 0;
        mbar_wait(&bars->drain, 0, &no_abort, g.status, kDevTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue warpgroups
    // Parameters into shared memory (GELU / bias: N bias values; LN: bias | gamma |
    // beta, NT each) by bulk copies that land while the first tile accumulates;
    // every epilogue thread waits for them (bounded) before its first tile.
    float* sparams = reinterpret_cast<float*>(smem + STAGES * kStage + kBarrierBytes +
                                              8 * epi_groups_per_tile<EPI>() * stage_words<EPI>() * 4);
    if (threadIdx.x == 64) {
      if (EPI == kEpiTokenizer) {
        mbar_arrive(&bars->params);  // no parameter copy: the epilogue reads them through L1
      } else if (EPI != kEpiResidualLN) {
        mbar_arrive_expect_tx(&bars->params, static_cast<uint32_t>(g.N) * 4u);
        bulk_load(sparams, g.bias, static_cast<uint32_t>(g.N) * 4u, &bars->params);
      } else {
        mbar_arrive_expect_tx(&bars->params, 3u * NT * 4u);
        bulk_load(sparams, g.bias, NT * 4u, &bars->params);
        bulk_load(sparams + NT, g.gamma, NT * 4u, &bars->params);
        bulk_load(sparams + 2 * NT, g.beta, NT * 4u, &bars->params);
      }
    }
    bool params_ready = false;
    constexpr int kSplit = epi_groups_per_tile<EPI>();
    constexpr int kCols = NT / kSplit;                      // columns per group
    const int grp = (warp - 2) >> 2;
    const uint32_t e = grp / kSplit;                        // takes local tiles with lt % 2 == e
    const int col0 = (grp % kSplit) * kCols;                // first tile column of this group
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    uint32_t* stage = reinterpret_cast<uint32_t*>(smem + STAGES * kStage + kBarrierBytes) + (warp - 2) * stage_words<EPI>();
    uint32_t lt = 0;
    bool ok = true;
    if (EPI == kEpiTokenizer) {
      // Both groups take every tile: group grp drains row sub-tile grp.
      for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x, ++lt) {
        const int64_t row = (t / g.n_tiles_n) * kTileM + grp * kGBM + (warp & 3) * 32 + lane;
        tokenizer_stage_pos(t % g.n_tiles_n, row, g, lane, reinterpret_cast<float*>(stage));
        if (!mbar_wait(&bars->acc_full[0], lt & 1, abort_flag, g.status, kDevTimeoutSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        epilogue_tokenizer(lane_base + grp * NT, t % g.n_tiles_n, row, g, lane, reinterpret_cast<float*>(stage),
                           &bars->acc_empty[0]);
      }
    }
    for (int64_t t = blockIdx.x; EPI != kEpiTokenizer && t < g.tiles && ok; t += gridDim.x, ++lt) {
      if ((lt & 1) != e) continue;
      const int32_t n0 = static_cast<int32_t>((t % g.n_tiles_n) * NT);
      const uint32_t acc = lane_base + e * NT + col0;
      const int64_t wrow0 = (t / g.n_tiles_n) * kGBM + (warp & 3) * 32;  // first row of this warp
      if (EPI != kEpiResidualLN) {
        if (!mbar_wait(&bars->acc_full[e], (lt >> 1) & 1, abort_flag, g.status, kDevTimeoutSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (!params_ready) {
          if (!mbar_wait(&bars->params, 0, abort_flag, g.status, kDevTimeoutSoftmax)) {
            ok = false;
            break;
          }
          params_ready = true;
        }
        epilogue_gelu<kCols, EPI == kEpiGelu>(acc, sparams + n0 + col0, stage, lane, g.out + n0 + col0, g.out_stride,
                                              wrow0, g.M,
                             &bars->acc_empty[e]);
      } else {
        // The residual rows are fetched into L2, and their first 32 columns
        // into shared memory, while the tile still accumulates.
        float* xbuf = reinterpret_cast<float*>(stage);
        if (wrow0 + lane < g.M) bulk_prefetch_l2(g.x + (wrow0 + lane) * g.x_stride, NT * 4);
        copy_x_chunk(xbuf, g.x, g.x_stride, wrow0, g.M, 0, lane);
        if (!mbar_wait(&bars->acc_full[e], (lt >> 1) & 1, abort_flag, g.status, kDevTimeoutSoftmax)) {
          cp_async_wait<0>();
          ok = false;
          break;
        }
        tc_fence_after();
        if (!params_ready) {
          if (!mbar_wait(&bars->params, 0, abort_flag, g.status, kDevTimeoutSoftmax)) {
            cp_async_wait<0>();
            ok = false;
            break;
          }
          params_ready = true;
        }
        epilogue_residual_ln<NT>(acc, sparams, xbuf, lane, g.x, g.x_stride, g.eps, g.h, g.h_stride, wrow0, g.M,
                                 &bars->acc_empty[e]);
      }
    }
  }

  if (threadIdx.x == 64) {  // the parameter copy has landed before the CTA exits
    volatile int32_t no_abort = 0;
    mbar_wait(&bars->params, 0, &no_abort, g.status, kDevTimeoutDrain);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// 2-D bf16 tensor map over rows x cols (row stride in elements), box 64 x box_rows, 128-byte swizzle.
bool make_map_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t row_stride,
                 uint32_t box_rows) {
  EncodeTiledFn enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kGBK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int NT, int STAGES, int EPI>
intp_status launch_gemm(const void* a, int64_t a_stride, const void* w, GemmArgs g, cudaStream_t stream) {
  if ((EPI != kEpiTokenizer && g.K % kGBK) || g.K % 8 || g.N % NT) return INTP_ERR_SHAPE;
  if (!aligned16(a) || !aligned16(w) || (a_stride * 2) % 16) return INTP_ERR_LAYOUT;
  CUtensorMap ma, mb;
  if (!make_map_2d(&ma, a, g.M, g.K, a_stride, kGBM) || !make_map_2d(&mb, w, g.N, g.K, g.K, NT))
    return INTP_ERR_LAYOUT;
  g.n_tiles_n = g.N / NT;
  constexpr int64_t kTileM = m_subtiles<EPI>() * kGBM;
  g.tiles = ((g.M + kTileM - 1) / kTileM) * g.n_tiles_n;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return INTP_ERR_LAUNCH;
  auto kernel = gemm_epilogue_kernel<NT, STAGES, EPI>;
  static_assert(sizeof(GemmBarriers<STAGES>) <= kBarrierBytes, "barrier block");
  const size_t params = EPI == kEpiTokenizer ? 0 : (EPI != kEpiResidualLN ? static_cast<size_t>(g.N) : 3 * NT);
  const size_t smem = 1024 + STAGES * (m_subtiles<EPI>() * kASlab + NT * kGBK * 2) + kBarrierBytes + 8 * epi_groups_per_tile<EPI>() * stage_words<EPI>() * 4 + params * 4;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return INTP_ERR_LAUNCH;
  const int64_t grid = g.tiles < sms ? g.tiles : sms;
  kernel<<<static_cast<unsigned>(grid), gemm_threads<EPI>(), smem, stream>>>(ma, mb, g);
  return cudaGetLastError() == cudaSuccess ? INTP_OK : INTP_ERR_LAUNCH;
}

bool device_is_sm100() {
  int dev = 0, major = 0;
  return cudaGetDevice(&dev) == cudaSuccess &&
         cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess && major == 10;
}

}  // namespace
}  // namespace intp

using namespace intp;

extern "C" INTP_API intp_status svit_linear_gelu(const void* a, int64_t a_stride, int64_t rows, int32_t in_features,
                                                 const void* weight, const float* bias, int32_t out_features,
                                                 void* out, int64_t out_stride, int32_t* status, void* stream) {
  if (rows < 0 || in_features < 1 || out_features < 1) return INTP_ERR_SHAPE;
  if (rows == 0) return INTP_OK;
  if (out_features > kMaxGeluN) return INTP_ERR_UNSUPPORTED;
  if (!a || !weight || !bias || !out || !status) return INTP_ERR_ARGUMENT;
  if (a_stride < in_features || out_stride < out_features || out_stride % 8 || !aligned16(out) || !aligned16(bias))
    return INTP_ERR_LAYOUT;
  if (!device_is_sm100()) return INTP_ERR_ARCH;
  GemmArgs g{};
  g.M = rows;
  g.N = out_features;
  g.K = in_features;
  g.bias = bias;
  g.out = static_cast<__nv_bfloat16*>(out);
  g.out_stride = out_stride;
  g.status = status;
  return launch_gemm<256, 3, kEpiGelu>(a, a_stride, weight, g, static_cast<cudaStream_t>(stream));
}

extern "C" INTP_API intp_status svit_linear_bias(const void* a, int64_t a_stride, int64_t rows, int32_t in_features,
                                                 const void* weight, const float* bias, int32_t out_features,
                                                 void* out, int64_t out_stride, int32_t* status, void* stream) {
  if (rows < 0 || in_features < 1 || out_features < 1) return INTP_ERR_SHAPE;
  if (rows == 0) return INTP_OK;
  if (out_features > kMaxGeluN) return INTP_ERR_UNSUPPORTED;
  if (!a || !weight || !bias || !out || !status) return INTP_ERR_ARGUMENT;
  if (a_stride < in_features || out_stride < out_features || out_stride % 8 || !aligned16(out) || !aligned16(bias))
    return INTP_ERR_LAYOUT;
  if (!device_is_sm100()) return INTP_ERR_ARCH;
  GemmArgs g{};
  g.M = rows;
  g.N = out_features;
  g.K = in_features;
  g.bias = bias;
  g.out = static_cast<__nv_bfloat16*>(out);
  g.out_stride = out_stride;
  g.status = status;
  return launch_gemm<192, 3, kEpiBias>(a, a_stride, weight, g, static_cast<cudaStream_t>(stream));
}

extern "C" INTP_API intp_status svit_linear_residual_layernorm(const void* a, int64_t a_stride, int64_t rows,
                                                               int32_t in_features, const void* weight,
                                                               const float* bias, int32_t dim, float* x,
                                                               int64_t x_stride, const float* gamma, const float* beta,
                                                               float eps, void* h, int64_t h_stride, int32_t* status,
                                                               void* stream) {
  if (rows < 0 || in_features < 1 || dim < 1) return INTP_ERR_SHAPE;
  if (rows == 0) return INTP_OK;
  if (!a || !weight || !bias || !x || !gamma || !beta || !h || !status) return INTP_ERR_ARGUMENT;
  if (dim != 192) return INTP_ERR_UNSUPPORTED;
  if (a_stride < in_features || x_stride < dim || h_stride < dim || x_stride % 4 || h_stride % 8 || !aligned16(x) ||
      !aligned16(h) || !aligned16(bias) || !aligned16(gamma) || !aligned16(beta))
    return INTP_ERR_LAYOUT;
  if (!device_is_sm100()) return INTP_ERR_ARCH;
  GemmArgs g{};
  g.M = rows;
  g.N = dim;
  g.K = in_features;
  g.bias = bias;
  g.x = x;
  g.x_stride = x_stride;
  g.gamma = gamma;
  g.beta = beta;
  g.eps = eps;
  g.h = static_cast<__nv_bfloat16*>(h);
  g.h_stride = h_stride;
  g.status = status;
  return launch_gemm<192, 3, kEpiResidualLN>(a, a_stride, weight, g, static_cast<cudaStream_t>(stream));
}

extern "C" INTP_API intp_status svit_tokenizer_gemm(const svit_embed_args* args, const void* patches,
                                                    int64_t patches_stride, int32_t features, const void* weight,
                                                    int32_t* status, void* stream) {
  if (!args || !patches || !weight || !status) return INTP_ERR_ARGUMENT;
  const svit_embed_args& a = *args;
  if (a.batch < 0 || a.patches < 1 || features < 8) return INTP_ERR_SHAPE;
  if (a.batch == 0) return INTP_OK;
  if (a.directions != kTokDirs || a.look_poses != kLookPoses || a.bases % (kTokTileN / kTokDirs) ||
      a.look_heads % (kTokTileN / kLookPoses) || a.bases < 1 || a.look_heads < 1)
    return INTP_ERR_UNSUPPORTED;
  if (a.values != nullptr || !a.look_pose || !a.x || !a.token_null || !a.direction_coef || !a.output_bias || !a.cls ||
      !a.pos_embed || !a.look_null)
    return INTP_ERR_ARGUMENT;
  if (features % 8 || patches_stride < features || !aligned16(a.look_pose) || !aligned16(a.x) ||
      !aligned16(a.pos_embed) || !aligned16(a.cls) || !aligned16(a.output_bias))
    return INTP_ERR_LAYOUT;
  if (!device_is_sm100()) return INTP_ERR_ARCH;
  GemmArgs g{};
  g.M = a.batch * a.patches;
  g.N = a.bases * kTokDirs + a.look_heads * kLookPoses;
  g.K = features;
  g.x = a.x;
  g.status = status;
  g.patches = static_cast<int32_t>(a.patches);
  g.tok_tiles = a.bases * kTokDirs / kTokTileN;
  g.token_null = a.token_null;
  g.direction_coef = a.direction_coef;
  g.output_bias = a.output_bias;
  g.cls = a.cls;
  g.pos_embed = a.pos_embed;
  g.look_null = a.look_null;
  g.look_pose = a.look_pose;
  g.look_heads = a.look_heads;
  return launch_gemm<kTokTileN, 3, kEpiTokenizer>(patches, patches_stride, weight, g,
                                                   static_cast<cudaStream_t>(stream));
}
