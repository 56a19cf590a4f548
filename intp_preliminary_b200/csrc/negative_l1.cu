// negative_l1.cu - negative L1 distance projection on CUDA cores (sm_100a).
//
//   out[m, p] = -sum_f |x[m, f] - w[p, f]|     (fp32 in, fp32 accumulate, fp32 out)
//
// Semantics: layers/triton_negative_l1.py:19-52 (Triton forward) and :233-241
// (`-torch.cdist(x, w, p=1)` on CPU).  This is not a contraction, so no tensor
// core applies: every (m, p, f) triple costs one subtract and one
// absolute-value add on the FP32 pipe, which bounds the kernel (the arithmetic
// intensity is ~200 op/B, far above the HBM ridge).
//
// nl1_vec_kernel (16-byte aligned rows, F % 4 == 0 - every shape of the
// reference): CTA tile 128 rows x 96 prototypes, 256 threads, thread tile
// 8 rows x 6 prototypes (rows ty + 16 i, prototypes tx + 16 j).  The feature
// axis streams in chunks of 32 through a 3-stage shared-memory ring filled by
// 16-byte cp.async copies (rows padded to 36 floats: the 128-bit reads of a
// quarter-warp land in 8 distinct bank groups).  Each 128-bit shared read
// feeds 24 (x) or 32 (w) subtract / |.|-add pairs.  Sums run over f in
// increasing order per (m, p), like the reference's loop.
// nl1_kernel: the scalar form for any other layout (odd F, unaligned rows).
#include <cstdint>
#include <cuda_runtime.h>
#include "sla_internal.h"

namespace intp {
namespace {

constexpr int TM = 8, TP = 4;          // thread tile
constexpr int GM = 16, GP = 16;        // thread grid (m, p)
constexpr int BMr = TM * GM;           // 128 rows
constexpr int BPr = TP * GP;           // 64 prototypes
constexpr int FC = 32;                 // feature chunk
constexpr int LD = FC + 1;             // padded smem row
constexpr int kThreads = GM * GP;      // 256

__global__ void __launch_bounds__(kThreads, 2)
nl1_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ out, int64_t rows,
           int64_t protos, int64_t features) {
  __shared__ float xs[BMr * LD];
  __shared__ float ws[BPr * LD];
  const int tid = threadIdx.x;
  const int tp = tid % GP, tm = tid / GP;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BMr;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * BPr;

  // Loader mapping: 8 threads per 32-float row segment (one float each x4 rows).
  // x tile: 128 rows x 32 feats = 4096 floats -> 16 per thread.
  // w tile:  64 rows x 32 feats = 2048 floats ->  8 per thread.
  const int lc = tid % FC;   // feature within chunk
  const int lr = tid / FC;   // 0..7
  float xr[BMr / 8], wr[BPr / 8];

  auto fetch = [&](int64_t f0) {
    const int64_t f = f0 + lc;
    const bool fok = f < features;
#pragma unroll
    for (int k = 0; k < BMr / 8; ++k) {
      const int64_t m = m0 + lr + 8 * k;
      xr[k] = (fok && m < rows) ? __ldg(x + m * features + f) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < BPr / 8; ++k) {
      const int64_t pp = p0 + lr + 8 * k;
      wr[k] = (fok && pp < protos) ? __ldg(w + pp * features + f) : 0.f;
    }
  };
  auto stash = [&]() {
#pragma unroll
    for (int k = 0; k < BMr / 8; ++k) xs[(lr + 8 * k) * LD + lc] = xr[k];
#pragma unroll
    for (int k = 0; k < BPr / 8; ++k) ws[(lr + 8 * k) * LD + lc] = wr[k];
  };

  float acc[TM][TP];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TP; ++j) acc[i][j] = 0.f;

  fetch(0);
  for (int64_t f0 = 0; f0 < features; f0 += FC) {
    __syncthreads();
    stash();
    __syncthreads();
    if (f0 + FC < features) fetch(f0 + FC);
#pragma unroll 8
    for (int f = 0; f < FC; ++f) {
      float xv[TM], wv[TP];
#pragma unroll
      for (int i = 0; i < TM; ++i) xv[i] = xs[(tm + GM * i) * LD + f];
#pragma unroll
      for (int j = 0; j < TP; ++j) wv[j] = ws[(tp + GP * j) * LD + f];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TP; ++j) acc[i][j] += fabsf(xv[i] - wv[j]);
    }
  }

#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t m = m0 + tm + GM * i;
    if (m >= rows) continue;
#pragma unroll
    for (int j = 0; j < TP; ++j) {
      const int64_t pp = p0 + tp + GP * j;
      if (pp < protos) out[m * protos + pp] = -acc[i][j];
    }
  }
}

// ------------------------------------------------------------ 16-byte form
constexpr int VTM = 8, VTP = 6;                 // thread tile
constexpr int VBM = VTM * 16, VBP = VTP * 16;   // 128 rows x 96 prototypes
constexpr int VFC = 32;                         // features per chunk
constexpr int VLD = VFC + 4;                    // padded smem row (floats)
constexpr int VStages = 3;
constexpr int VStageFloats = (VBM + VBP) * VLD;

__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  const int bytes = valid ? 16 : 0;  // src-size 0: the 16 bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(kThreads, 2)
nl1_vec_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ out, int64_t rows,
               int64_t protos, int64_t features) {
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * VBM;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * VBP;
  const int64_t chunks = (features + VFC - 1) / VFC;

  // Copies of one chunk: (128 + 96) rows x 8 units of 16 bytes = 1792 units, 7 per thread.
  auto load_chunk = [&](int64_t c, int stage) {
    float* xs = smem + stage * VStageFloats;
    float* ws = xs + VBM * VLD;
    const int64_t f0 = c * VFC;
#pragma unroll
    for (int k = 0; k < 7; ++k) {
      const int u = tid + k * kThreads;  // 0..1791
      const int r = u >> 3, q = u & 7;
      const int64_t f = f0 + 4 * q;
      if (r < VBM) {
        const int64_t m = m0 + r;
        const bool ok = m < rows && f < features;
        cp_async16(xs + r * VLD + 4 * q, ok ? x + m * features + f : x, ok);
      } else {
        const int64_t pp = p0 + (r - VBM);
        const bool ok = pp < protos && f < features;
        cp_async16(ws + (r - VBM) * VLD + 4 * q, ok ? w + pp * features + f : w, ok);
      }
    }
  };

  float acc[VTM][VTP];
#pragma unroll
  for (int i = 0; i < VTM; ++i)
#pragma unroll
    for (int j = 0; j < VTP; ++j) acc[i][j] = 0.f;

#pragma unroll
  for (int s = 0; s < VStages - 1; ++s) {
    if (s < chunks) load_chunk(s, s);
    cp_async_commit();
  }
  for (int64_t c = 0; c < chunks; ++c) {
    cp_async_wait<VStages - 2>();  // chunk c has landed (this thread's copies)
    __syncthreads();               // ... and everyone's; stage (c - 1) % S is free again
    if (c + VStages - 1 < chunks) load_chunk(c + VStages - 1, static_cast<int>((c + VStages - 1) % VStages));
    cp_async_commit();
    const float* xs = smem + static_cast<int>(c % VStages) * VStageFloats;
    const float* ws = xs + VBM * VLD;
#pragma unroll 2
    for (int f = 0; f < VFC; f += 4) {
      float4 xv[VTM], wv[VTP];
#pragma unroll
      for (int i = 0; i < VTM; ++i) xv[i] = *reinterpret_cast<const float4*>(xs + (ty + 16 * i) * VLD + f);
#pragma unroll
      for (int j = 0; j < VTP; ++j) wv[j] = *reinterpret_cast<const float4*>(ws + (tx + 16 * j) * VLD + f);
#pragma unroll
      for (int i = 0; i < VTM; ++i)
#pragma unroll
        for (int j = 0; j < VTP; ++j) {
          float a = acc[i][j];
          a += fabsf(xv[i].x - wv[j].x);
          a += fabsf(xv[i].y - wv[j].y);
          a += fabsf(xv[i].z - wv[j].z);
          a += fabsf(xv[i].w - wv[j].w);
          acc[i][j] = a;
        }
    }
  }

#pragma unroll
  for (int i = 0; i < VTM; ++i) {
    const int64_t m = m0 + ty + 16 * i;
    if (m >= rows) continue;
#pragma unroll
    for (int j = 0; j < VTP; ++j) {
      const int64_t pp = p0 + tx + 16 * j;
      if (pp < protos) out[m * protos + pp] = -acc[i][j];
    }
  }
}

}  // namespace

int32_t launch_nl1(const float* x, const float* w, float* out, int64_t rows, int64_t protos, int64_t features,
                   cudaStream_t stream) {
  if (rows == 0 || protos == 0) return 0;
  if (features == 0) return cudaMemsetAsync(out, 0, sizeof(float) * rows * protos, stream) == cudaSuccess ? 0 : 6;
  const bool vec = features % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(w) % 16 == 0;
  if (vec) {
    const int64_t gx = (protos + VBP - 1) / VBP, gy = (rows + VBM - 1) / VBM;
    if (gx > 2147483647LL || gy > 65535LL) return 8;
    const size_t smem = sizeof(float) * VStages * VStageFloats;  // 96.8 KB: two CTAs per SM
    if (cudaFuncSetAttribute(nl1_vec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return 6;
    nl1_vec_kernel<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), kThreads, smem, stream>>>(
        x, w, out, rows, protos, features);
    return cudaGetLastError() == cudaSuccess ? 0 : 6;
  }
  const int64_t gx = (protos + BPr - 1) / BPr, gy = (rows + BMr - 1) / BMr;
  if (gx > 2147483647LL || gy > 65535LL) return 8;
  nl1_kernel<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), kThreads, 0, stream>>>(x, w, out, rows,
                                                                                                  protos, features);
  return cudaGetLastError() == cudaSuccess ? 0 : 6;
}

}  // namespace intp
