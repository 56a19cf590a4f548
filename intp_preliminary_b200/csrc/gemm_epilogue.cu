// gemm_epilogue.cu - tcgen05 GEMM with the transformer block's element-wise
// work fused into its epilogue (C ABI in include/intp_share_vit.h).
//
//   C[M, N] = A[M, K] W[N, K]^T + bias     (bf16 operands, fp32 accumulation in TMEM)
//   GELU epilogue:      out = bf16(GELU_erf(C))                       (MLP fc1)
//   residual + LN:      x += C (fp32);  h = bf16(LayerNorm(x))         (attention proj, MLP fc2)
// so the MLP's 768-wide activation is written once (by fc1, already
// activated) and the residual stream is read and written once per sub-block,
// with no separate GELU or add + LayerNorm pass (layers/mini_vit.py:138-170).
//
// CTA (one per SM, persistent over 128-row x NT-column tiles): warp 0 issues
// TMA loads of 64-wide K slabs of A and W into a STAGES-deep ring (128-byte
// swizzle); warp 1 issues tcgen05.mma (M = 128, N = NT, K = 16 per
// instruction) into one of two TMEM accumulators; warpgroups 1 and 2 (warps
// 4-7, 8-11) take alternate tiles and run the epilogue from TMEM, one row per
// thread, while the next tile accumulates in the other buffer.  Every wait is
// bounded (sm100_ptx.cuh).
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
constexpr int kGemmThreads = 384;                  // warps 0 (TMA), 1 (MMA), 2-3 idle, 4-11 epilogue
constexpr int kEpiGelu = 0, kEpiResidualLN = 1;
constexpr int kStageWords = 32 * 33;     // per epilogue warp: 32 rows x 32 columns, pitch 33
constexpr uint32_t kBarrierBytes = 256;  // room reserved for the barrier block

struct GemmArgs {
  int64_t M;
  int32_t N, K;
  int32_t n_tiles_n;   // N / NT
  int64_t tiles;       // ceil(M / 128) * n_tiles_n
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
};

template <int STAGES>
struct GemmBarriers {
  uint64_t full[STAGES], empty[STAGES];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int32_t abort;
};

// GELU with the exact error function, as nn.GELU() computes it.
__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }

template <int NT, int STAGES, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_epilogue_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const GemmArgs g) {
  constexpr uint32_t kBSlab = NT * kGBK * 2;
  constexpr uint32_t kStage = kASlab + kBSlab;
  constexpr uint32_t kTmemCols = 2 * NT <= 256 ? 256 : 512;
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
      mbar_init(&bars->acc_empty[b], 4);
    }
    mbar_init(&bars->drain, 1);
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
  const int n_slabs = g.K / kGBK;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      uint32_t loads = 0, stage = 0, phase = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
        const int32_t m0 = static_cast<int32_t>((t / g.n_tiles_n) * kGBM);
        const int32_t n0 = static_cast<int32_t>((t % g.n_tiles_n) * NT);
        for (int ks = 0; ks < n_slabs; ++ks) {
          if (loads >= STAGES &&
              !mbar_wait(&bars->empty[stage], phase ^ 1u, abort_flag, g.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + stage * kStage;
          mbar_arrive_expect_tx(&bars->full[stage], kStage);
          tma_load_2d(dst, &tm_a, &bars->full[stage], ks * kGBK, m0);
          tma_load_2d(dst + kASlab, &tm_b, &bars->full[stage], ks * kGBK, n0);
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
      const uint64_t b_desc = smem_desc_sw128(smem_u32(smem + kASlab), 16, 1024);
      uint32_t stage = 0, phase = 0, lt = 0;
      bool ok = true, issued = false;
      for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x, ++lt) {
        const uint32_t buf = lt & 1;
        if (lt >= 2 &&
            !mbar_wait(&bars->acc_empty[buf], ((lt - 2) >> 1) & 1, abort_flag, g.status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int ks = 0; ks < n_slabs; ++ks) {
          if (!mbar_wait(&bars->full[stage], phase, abort_flag, g.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kGBK / 16; ++kk)
            mma_ss(tmem + buf * NT, a_desc + ((stage * kStage + kk * 32) >> 4),
                   b_desc + ((stage * kStage + kk * 32) >> 4), idesc, (ks > 0 || kk > 0) ? 1u : 0u);
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
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue warpgroups
    const uint32_t e = (warp - 4) >> 2;   // warpgroup: takes local tiles with lt % 2 == e
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    uint32_t* stage = reinterpret_cast<uint32_t*>(smem + STAGES * kStage + kBarrierBytes) + (warp - 4) * kStageWords;
    uint32_t lt = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x, ++lt) {
      if ((lt & 1) != e) continue;
      if (!mbar_wait(&bars->acc_full[e], (lt >> 1) & 1, abort_flag, g.status, kDevTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int32_t n0 = static_cast<int32_t>((t % g.n_tiles_n) * NT);
      const uint32_t acc = lane_base + e * NT;
      // Warp-cooperative global traffic: a chunk of 32 columns of the warp's 32
      // rows is staged in `stage` (row pitch 33 words: conflict free both ways)
      // and moved one row per instruction, 32 lanes on 32 consecutive columns.
      const int64_t wrow0 = (t / g.n_tiles_n) * kGBM + (warp & 3) * 32;  // first row of this warp
      if (EPI == kEpiGelu) {
#pragma unroll 1
        for (int c = 0; c < NT; c += 32) {
          uint32_t r0[16], r1[16];
          tmem_ld16(acc + c, r0);
          tmem_ld16(acc + c + 16, r1);
          tmem_wait_ld();
          reg_fence16(r0);
          reg_fence16(r1);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int n = n0 + c + 2 * i;
            stage[lane * 33 + i] = pack_bf16x2(gelu_erf(__uint_as_float(r0[2 * i]) + __ldg(g.bias + n)),
                                               gelu_erf(__uint_as_float(r0[2 * i + 1]) + __ldg(g.bias + n + 1)));
            stage[lane * 33 + 8 + i] =
                pack_bf16x2(gelu_erf(__uint_as_float(r1[2 * i]) + __ldg(g.bias + n + 16)),
                            gelu_erf(__uint_as_float(r1[2 * i + 1]) + __ldg(g.bias + n + 17)));
          }
          __syncwarp();
          // 16 words (32 bf16) per row: lanes 0-15 row i, lanes 16-31 row i + 1
#pragma unroll 4
          for (int i = 0; i < 32; i += 2) {
            const int rr = i + (lane >> 4);
            const int64_t m = wrow0 + rr;
            if (m < g.M)
              reinterpret_cast<uint32_t*>(g.out + m * g.out_stride + n0 + c)[lane & 15] = stage[rr * 33 + (lane & 15)];
          }
          __syncwarp();
        }
      } else {
        // pass 1: v = C + bias + x; x written back; v kept in TMEM; row sum
        float sum = 0.f;
        float* fstage = reinterpret_cast<float*>(stage);
#pragma unroll 1
        for (int c = 0; c < NT; c += 32) {
          uint32_t r0[16], r1[16];
          tmem_ld16(acc + c, r0);
          tmem_ld16(acc + c + 16, r1);
          tmem_wait_ld();
          reg_fence16(r0);
          reg_fence16(r1);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            fstage[lane * 33 + i] = __uint_as_float(r0[i]) + __ldg(g.bias + c + i);
            fstage[lane * 33 + 16 + i] = __uint_as_float(r1[i]) + __ldg(g.bias + c + 16 + i);
          }
          __syncwarp();
#pragma unroll 4
          for (int i = 0; i < 32; ++i) {
            const int64_t m = wrow0 + i;
            if (m < g.M) {
              float* xp = g.x + m * g.x_stride + c + lane;
              const float v = fstage[i * 33 + lane] + *xp;
              *xp = v;
              fstage[i * 33 + lane] = v;
            }
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            r0[i] = __float_as_uint(fstage[lane * 33 + i]);
            r1[i] = __float_as_uint(fstage[lane * 33 + 16 + i]);
            sum += __uint_as_float(r0[i]) + __uint_as_float(r1[i]);
          }
          __syncwarp();
          tmem_st16(acc + c, r0);
          tmem_st16(acc + c + 16, r1);
        }
        tmem_wait_st();
        const float mean = sum * (1.f / NT);
        // pass 2: variance about the mean
        float var = 0.f;
#pragma unroll 1
        for (int c = 0; c < NT; c += 16) {
          uint32_t r[16];
          tmem_ld16(acc + c, r);
          tmem_wait_ld();
          reg_fence16(r);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float d = __uint_as_float(r[i]) - mean;
            var = fmaf(d, d, var);
          }
        }
        const float rstd = rsqrtf(var * (1.f / NT) + g.eps);
        // pass 3: h = bf16((v - mean) * rstd * gamma + beta), staged like the GELU output
#pragma unroll 1
        for (int c = 0; c < NT; c += 32) {
          uint32_t r0[16], r1[16];
          tmem_ld16(acc + c, r0);
          tmem_ld16(acc + c + 16, r1);
          tmem_wait_ld();
          reg_fence16(r0);
          reg_fence16(r1);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int n = c + 2 * i;
            stage[lane * 33 + i] = pack_bf16x2(
                fmaf((__uint_as_float(r0[2 * i]) - mean) * rstd, __ldg(g.gamma + n), __ldg(g.beta + n)),
                fmaf((__uint_as_float(r0[2 * i + 1]) - mean) * rstd, __ldg(g.gamma + n + 1), __ldg(g.beta + n + 1)));
            stage[lane * 33 + 8 + i] = pack_bf16x2(
                fmaf((__uint_as_float(r1[2 * i]) - mean) * rstd, __ldg(g.gamma + n + 16), __ldg(g.beta + n + 16)),
                fmaf((__uint_as_float(r1[2 * i + 1]) - mean) * rstd, __ldg(g.gamma + n + 17), __ldg(g.beta + n + 17)));
          }
          __syncwarp();
#pragma unroll 4
          for (int i = 0; i < 32; i += 2) {
            const int rr = i + (lane >> 4);
            const int64_t m = wrow0 + rr;
            if (m < g.M) reinterpret_cast<uint32_t*>(g.h + m * g.h_stride + c)[lane & 15] = stage[rr * 33 + (lane & 15)];
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[e]);
    }
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
  if (g.K % kGBK || g.N % NT) return INTP_ERR_SHAPE;
  if (!aligned16(a) || !aligned16(w) || (a_stride * 2) % 16) return INTP_ERR_LAYOUT;
  CUtensorMap ma, mb;
  if (!make_map_2d(&ma, a, g.M, g.K, a_stride, kGBM) || !make_map_2d(&mb, w, g.N, g.K, g.K, NT))
    return INTP_ERR_LAYOUT;
  g.n_tiles_n = g.N / NT;
  g.tiles = ((g.M + kGBM - 1) / kGBM) * g.n_tiles_n;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return INTP_ERR_LAUNCH;
  auto kernel = gemm_epilogue_kernel<NT, STAGES, EPI>;
  static_assert(sizeof(GemmBarriers<STAGES>) <= kBarrierBytes, "barrier block");
  const size_t smem = 1024 + STAGES * (kASlab + NT * kGBK * 2) + kBarrierBytes + 8 * kStageWords * 4;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return INTP_ERR_LAUNCH;
  const int64_t grid = g.tiles < sms ? g.tiles : sms;
  kernel<<<static_cast<unsigned>(grid), kGemmThreads, smem, stream>>>(ma, mb, g);
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
  if (!a || !weight || !bias || !out || !status) return INTP_ERR_ARGUMENT;
  if (a_stride < in_features || out_stride < out_features || out_stride % 8 || !aligned16(out))
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
      !aligned16(h))
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
  return launch_gemm<192, 4, kEpiResidualLN>(a, a_stride, weight, g, static_cast<cudaStream_t>(stream));
}
