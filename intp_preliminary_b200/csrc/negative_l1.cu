// negative_l1.cu - negative L1 distance projection on CUDA cores (sm_100a).
//
//   out[m, p] = -sum_f |x[m, f] - w[p, f]|     (fp32 in, fp32 accumulate, fp32 out)
//
// Semantics: layers/triton_negative_l1.py:19-52 (Triton forward) and :233-241
// (`-torch.cdist(x, w, p=1)` on CPU).  This is not a contraction, so no tensor
// core applies: every (m, p, f) triple costs one subtract and one
// absolute-value add.  The kernel is FP32-issue bound; it is register blocked
// so each shared-memory value feeds several FP32 ops:
//   CTA tile 128 rows x 64 prototypes, 256 threads, thread tile 8 x 4,
//   feature axis streamed in chunks of 32 through shared memory with a
//   register-staged prefetch of the next chunk.
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

}  // namespace

int32_t launch_nl1(const float* x, const float* w, float* out, int64_t rows, int64_t protos, int64_t features,
                   cudaStream_t stream) {
  if (rows == 0 || protos == 0) return 0;
  const int64_t gx = (protos + BPr - 1) / BPr, gy = (rows + BMr - 1) / BMr;
  if (gx > 2147483647LL || gy > 65535LL) return 8;
  if (features == 0) return cudaMemsetAsync(out, 0, sizeof(float) * rows * protos, stream) == cudaSuccess ? 0 : 6;
  nl1_kernel<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), kThreads, 0, stream>>>(x, w, out, rows,
                                                                                                  protos, features);
  return cudaGetLastError() == cudaSuccess ? 0 : 6;
}

}  // namespace intp
