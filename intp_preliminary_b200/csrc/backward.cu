// backward.cu - gradients of the structured Look attention and of the
// negative-L1 projection (CUDA cores, fp32 accumulation).
//
// Look attention (layers/triton_structured_look_attention.py:172-292 and
// :341-409 of the reference, which materialises P and dS as B*H*N^2 tensors and
// then runs batched matmuls): here flash-style, from the forward's LSE, with no
// N x N tensor except the requested dense-bias gradient itself:
//   P = exp(S - lse),  dP = dO V^T,  dS = P (dP - rowsum(dO * O)),
//   dQ = scale dS K,  dK = scale dS^T Q,  dV = P^T dO,
//   dbias = dS[1:,1:]  ->  dpose = sum_k dbias * fields,
//                          dfields = sum_b pose * dbias,  ddense = dbias.
// Kernel rows_kernel (one CTA per 16 query rows) produces dQ and the bias
// gradients; cols_kernel (one CTA per 16 keys) produces dK and dV; both
// recompute S and P.  In SLOTS mode the per-slot gradient of each query row is
// a shared-memory histogram of dS over the row's slots.
//
// Negative L1 (layers/triton_negative_l1.py:55-154): with s = sign(x - w)
// (sign(0) = 0), grad_x[m,f] = -sum_p g[m,p] s,  grad_w[p,f] = sum_m g[m,p] s.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "sla_internal.h"

namespace intp {
namespace {

constexpr int kRows = 16;   // rows (queries or keys) per CTA
constexpr int kWarps = 4;
constexpr int kRowsPerWarp = kRows / kWarps;
constexpr int kChunk = 32;  // streamed keys (rows_kernel) or queries (cols_kernel) per step
constexpr int kMaxDim = 128;
constexpr int kMaxBwdPoses = 253;

__device__ __forceinline__ float load_any(const void* p, int64_t idx, int32_t dtype) {
  switch (dtype) {
    case 1: return __half2float(static_cast<const __half*>(p)[idx]);
    case 2: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
    default: return static_cast<const float*>(p)[idx];
  }
}

// Look (+ dense) bias of pair (i, kj), both >= 1.  *slot receives the pair's
// slot in SLOTS mode (-1 when it has none).
__device__ __forceinline__ float pair_bias(const SlaParams& p, int64_t b, int64_t h, int64_t i, int64_t kj,
                                           int64_t n_kt64, int* slot) {
  const int64_t pq = i - 1, pk = kj - 1;
  float bias = 0.f;
  *slot = -1;
  if (p.bias_mode == 1) {
    for (int64_t pp = 0; pp < p.poses; ++pp) {
      const float w = load_any(p.pose, b * p.pose_stride[0] + pq * p.pose_stride[1] + h * p.pose_stride[2] +
                                           pp * p.pose_stride[3],
                               p.pose_dtype);
      const float f = load_any(p.fields, h * p.fields_stride[0] + pp * p.fields_stride[1] + pq * p.fields_stride[2] +
                                             pk * p.fields_stride[3],
                               p.fields_dtype);
      bias = fmaf(w, f, bias);
    }
  } else if (p.bias_mode == 2) {
    const int64_t qt = i >> 7, kt = kj >> 6;
    const int64_t off = (qt * n_kt64 + kt) * 8192 + ((kj & 63) >> 4) * 2048 + (i & 127) * 16 + (kj & 15);
    const int s = p.slots_packed[off];
    if (s < p.poses) {
      *slot = s;
      bias = load_any(p.pose, b * p.pose_stride[0] + pq * p.pose_stride[1] + h * p.pose_stride[2] +
                                  s * p.pose_stride[3],
                      p.pose_dtype);
    }
  }
  if (p.dense != nullptr)
    bias += load_any(p.dense, b * p.dense_stride[0] + h * p.dense_stride[1] + pq * p.dense_stride[2] +
                                  pk * p.dense_stride[3],
                     p.dense_dtype);
  return bias;
}

// delta[b,h,i] = sum_d dO[i,d] * O[i,d]; one warp per row.
__global__ void __launch_bounds__(256) delta_kernel(const SlaBwdParams bp) {
  const SlaParams& p = bp.f;
  const int64_t rows = p.batch * p.heads * p.seq;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t i = row % p.seq, bh = row / p.seq, h = bh % p.heads, b = bh / p.heads;
  float s = 0.f;
  for (int d = lane; d < p.head_dim; d += 32) {
    const float go = load_any(bp.grad_out, b * bp.grad_out_stride[0] + h * bp.grad_out_stride[1] +
                                               i * bp.grad_out_stride[2] + d * bp.grad_out_stride[3],
                              p.dtype);
    const float o = load_any(p.out, b * p.out_stride[0] + h * p.out_stride[1] + i * p.out_stride[2] +
                                        d * p.out_stride[3],
                             p.dtype);
    s = fmaf(go, o, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) bp.delta[row] = s;
}

// Shared-memory row layout: head_dim padded to D4 = a multiple of 4 (zeros
// past D) so rows are read as float4, and a row stride Dp with Dp / 4 odd, so
// that the 8 lanes of each quarter-warp reading 16 bytes of 8 different rows
// hit 8 different 4-bank groups.
__host__ __device__ constexpr int padded_dim(int D) { return (D + 3) & ~3; }
__host__ __device__ constexpr int row_stride(int D) {
  return (padded_dim(D) / 4) % 2 ? padded_dim(D) : padded_dim(D) + 4;
}

// Stages `rows` rows of a (B,H,N,D) tensor starting at r0 into smem as fp32
// (row stride Dp; columns D .. D4-1 and rows past N written as 0).
__device__ __forceinline__ void stage_rows(float* dst, int rows, int Dp, const void* src, const int64_t* st,
                                           int32_t dtype, int64_t b, int64_t h, int64_t r0, int64_t N, int D) {
  const int D4 = padded_dim(D);
  for (int idx = threadIdx.x; idx < rows * D4; idx += blockDim.x) {
    const int r = idx / D4, d = idx % D4;
    const int64_t i = r0 + r;
    dst[r * Dp + d] = i < N && d < D ? load_any(src, b * st[0] + h * st[1] + i * st[2] + d * st[3], dtype) : 0.f;
  }
}

// s[r] += a[r] . x, t[r] += c[r] . y over the padded head dimension for the
// warp's kRowsPerWarp rows: x, y are this lane's rows (float4 reads), a[r],
// c[r] the rows shared by the warp (broadcast float4 reads).  The sums run over
// d in order, one fma per element, as a scalar loop would.
__device__ __forceinline__ void dot_rows(float (&s)[kRowsPerWarp], float (&t)[kRowsPerWarp], const float* a0,
                                         const float* c0, int row_stride_a, const float* x, const float* y, int D4) {
  for (int e = 0; e < D4; e += 4) {
    const float4 xx = *reinterpret_cast<const float4*>(x + e), yy = *reinterpret_cast<const float4*>(y + e);
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const float4 aa = *reinterpret_cast<const float4*>(a0 + r * row_stride_a + e);
      const float4 cc = *reinterpret_cast<const float4*>(c0 + r * row_stride_a + e);
      s[r] = fmaf(aa.x, xx.x, s[r]);
      s[r] = fmaf(aa.y, xx.y, s[r]);
      s[r] = fmaf(aa.z, xx.z, s[r]);
      s[r] = fmaf(aa.w, xx.w, s[r]);
      t[r] = fmaf(cc.x, yy.x, t[r]);
      t[r] = fmaf(cc.y, yy.y, t[r]);
      t[r] = fmaf(cc.z, yy.z, t[r]);
      t[r] = fmaf(cc.w, yy.w, t[r]);
    }
  }
}

// dQ, dpose / dslot values, dfields, ddense for 16 query rows of one (b, h).
// TD = head_dim / 32 rounded up (1, 2 or 4): the per-lane accumulator width.
// Five CTAs per SM (96 registers) keep more warps in flight for the per-pair
// global loads of the Look lookup.
template <int TD>
__global__ void __launch_bounds__(kWarps * 32, 5) rows_kernel(const SlaBwdParams bp) {
  const SlaParams& p = bp.f;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = blockIdx.z, h = blockIdx.y, row0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int64_t N = p.seq, Np = N - 1;
  const int D = static_cast<int>(p.head_dim), D4 = padded_dim(D), Dp = row_stride(D);
  const int P = static_cast<int>(p.poses);
  const int64_t n_kt64 = (N + 63) / 64;
  extern __shared__ __align__(16) float smem[];
  float* q_s = smem;                  // kRows x Dp
  float* go_s = q_s + kRows * Dp;     // kRows x Dp
  float* k_s = go_s + kRows * Dp;     // kChunk x Dp
  float* v_s = k_s + kChunk * Dp;     // kChunk x Dp
  float* ds_tile = v_s + kChunk * Dp; // kRows x kChunk: dS rows of each warp
  float* dpose_s = ds_tile + kRows * kChunk;  // kRows x P (bias modes 1 and 2)
  stage_rows(q_s, kRows, Dp, p.q, p.q_stride, p.dtype, b, h, row0, N, D);
  stage_rows(go_s, kRows, Dp, bp.grad_out, bp.grad_out_stride, p.dtype, b, h, row0, N, D);
  if (p.bias_mode != 0)
    for (int idx = threadIdx.x; idx < kRows * P; idx += blockDim.x) dpose_s[idx] = 0.f;

  float lse[kRowsPerWarp], dlt[kRowsPerWarp], acc[kRowsPerWarp][TD];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int64_t i = row0 + warp * kRowsPerWarp + r;
    const int64_t bhi = (b * p.heads + h) * N + i;
    lse[r] = i < N ? p.lse[bhi] : 0.f;
    dlt[r] = i < N ? bp.delta[bhi] : 0.f;
#pragma unroll
    for (int t = 0; t < TD; ++t) acc[r][t] = 0.f;
  }

  for (int64_t key0 = 0; key0 < N; key0 += kChunk) {
    __syncthreads();
    stage_rows(k_s, kChunk, Dp, p.k, p.k_stride, p.dtype, b, h, key0, N, D);
    stage_rows(v_s, kChunk, Dp, p.v, p.v_stride, p.dtype, b, h, key0, N, D);
    __syncthreads();
    const int64_t kj = key0 + lane;
    const bool key_ok = kj < N;
    // S and dP of this lane's key against the warp's rows, together
    float sv[kRowsPerWarp], dpv[kRowsPerWarp], dsv[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) sv[r] = dpv[r] = 0.f;
    dot_rows(sv, dpv, q_s + warp * kRowsPerWarp * Dp, go_s + warp * kRowsPerWarp * Dp, Dp, k_s + lane * Dp,
             v_s + lane * Dp, D4);
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int rr = warp * kRowsPerWarp + r;
      const int64_t i = row0 + rr;
      dsv[r] = 0.f;
      if (i >= N) continue;  // warp-uniform
      float s = sv[r] * p.scale;
      const float dp = dpv[r];
      int slot = -1;
      const bool look = key_ok && i > 0 && kj > 0;
      if (look) s += pair_bias(p, b, h, i, kj, n_kt64, &slot);
      const float prob = key_ok ? expf(s - lse[r]) : 0.f;
      const float ds = prob * (dp - dlt[r]);
      dsv[r] = ds;
      if (!look) continue;
      const int64_t pq = i - 1, pk = kj - 1;
      if (bp.grad_dense != nullptr) bp.grad_dense[((b * p.heads + h) * Np + pq) * Np + pk] = ds;
      if (p.bias_mode == 2) {
        if (slot >= 0) atomicAdd(&dpose_s[rr * P + slot], ds);
      } else if (p.bias_mode == 1) {
        for (int pp = 0; pp < P; ++pp) {
          const float f = load_any(p.fields, h * p.fields_stride[0] + pp * p.fields_stride[1] +
                                                 pq * p.fields_stride[2] + pk * p.fields_stride[3],
                                   p.fields_dtype);
          atomicAdd(&dpose_s[rr * P + pp], ds * f);
          if (bp.grad_fields != nullptr) {
            const float w = load_any(p.pose, b * p.pose_stride[0] + pq * p.pose_stride[1] + h * p.pose_stride[2] +
                                                 pp * p.pose_stride[3],
                                     p.pose_dtype);
            atomicAdd(&bp.grad_fields[((h * P + pp) * Np + pq) * Np + pk], w * ds);
          }
        }
      }
    }
    // dQ += dS K (scale applied at the end): the warp's dS rows go through a
    // shared tile read four keys at a time (broadcast), each K value is read
    // once for the warp's rows
    float* ds_w = ds_tile + warp * kRowsPerWarp * kChunk;
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) ds_w[r * kChunk + lane] = dsv[r];
    __syncwarp();
    for (int j0 = 0; j0 < kChunk; j0 += 4) {
      float4 d4[kRowsPerWarp];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) d4[r] = *reinterpret_cast<const float4*>(ds_w + r * kChunk + j0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float kv[TD];
#pragma unroll
        for (int t = 0; t < TD; ++t) {
          const int d = lane + 32 * t;
          kv[t] = d < D ? k_s[(j0 + u) * Dp + d] : 0.f;
        }
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
          const float dsj = u == 0 ? d4[r].x : u == 1 ? d4[r].y : u == 2 ? d4[r].z : d4[r].w;
#pragma unroll
          for (int t = 0; t < TD; ++t) acc[r][t] = fmaf(dsj, kv[t], acc[r][t]);
        }
      }
    }
    __syncwarp();
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int64_t i = row0 + warp * kRowsPerWarp + r;
    if (i >= N || bp.grad_q == nullptr) continue;
#pragma unroll
    for (int t = 0; t < TD; ++t) {
      const int d = lane + 32 * t;
      if (d < D) bp.grad_q[(((b * p.heads + h) * N) + i) * D + d] = acc[r][t] * p.scale;
    }
  }
  if (p.bias_mode != 0 && bp.grad_pose != nullptr) {
    for (int idx = threadIdx.x; idx < kRows * P; idx += blockDim.x) {
      const int rr = idx / P, pp = idx % P;
      const int64_t i = row0 + rr;
      if (i >= 1 && i < N) bp.grad_pose[((b * Np + (i - 1)) * p.heads + h) * P + pp] = dpose_s[idx];
    }
  }
}

// dK, dV for 16 keys of one (b, h): streams query chunks.
template <int TD>
__global__ void __launch_bounds__(kWarps * 32, 5) cols_kernel(const SlaBwdParams bp) {
  const SlaParams& p = bp.f;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = blockIdx.z, h = blockIdx.y, key0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int64_t N = p.seq;
  const int D = static_cast<int>(p.head_dim), D4 = padded_dim(D), Dp = row_stride(D);
  const int64_t n_kt64 = (N + 63) / 64;
  extern __shared__ __align__(16) float smem[];
  float* k_s = smem;                  // kRows x Dp
  float* v_s = k_s + kRows * Dp;      // kRows x Dp
  float* q_s = v_s + kRows * Dp;      // kChunk x Dp
  float* go_s = q_s + kChunk * Dp;    // kChunk x Dp
  float* p_tile = go_s + kChunk * Dp;       // kRows x kChunk: P rows of each warp
  float* ds_tile = p_tile + kRows * kChunk;  // kRows x kChunk: dS rows of each warp
  float* lse_s = ds_tile + kRows * kChunk;   // kChunk
  float* dlt_s = lse_s + kChunk;             // kChunk
  stage_rows(k_s, kRows, Dp, p.k, p.k_stride, p.dtype, b, h, key0, N, D);
  stage_rows(v_s, kRows, Dp, p.v, p.v_stride, p.dtype, b, h, key0, N, D);

  float dk[kRowsPerWarp][TD], dv[kRowsPerWarp][TD];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int t = 0; t < TD; ++t) dk[r][t] = dv[r][t] = 0.f;

  for (int64_t q0 = 0; q0 < N; q0 += kChunk) {
    __syncthreads();
    stage_rows(q_s, kChunk, Dp, p.q, p.q_stride, p.dtype, b, h, q0, N, D);
    stage_rows(go_s, kChunk, Dp, bp.grad_out, bp.grad_out_stride, p.dtype, b, h, q0, N, D);
    if (threadIdx.x < kChunk) {
      const int64_t i = q0 + threadIdx.x;
      const int64_t bhi = (b * p.heads + h) * N + i;
      lse_s[threadIdx.x] = i < N ? p.lse[bhi] : 0.f;
      dlt_s[threadIdx.x] = i < N ? bp.delta[bhi] : 0.f;
    }
    __syncthreads();
    const int64_t i = q0 + lane;  // this lane's query
    const bool q_ok = i < N;
    // S and dP of this lane's query against the warp's keys, together
    float sv[kRowsPerWarp], dpv[kRowsPerWarp], pv[kRowsPerWarp], dsv[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) sv[r] = dpv[r] = 0.f;
    dot_rows(sv, dpv, k_s + warp * kRowsPerWarp * Dp, v_s + warp * kRowsPerWarp * Dp, Dp, q_s + lane * Dp,
             go_s + lane * Dp, D4);
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int64_t kj = key0 + warp * kRowsPerWarp + r;
      pv[r] = dsv[r] = 0.f;
      if (kj >= N) continue;  // warp-uniform
      float s = sv[r] * p.scale;
      int slot;
      if (q_ok && i > 0 && kj > 0) s += pair_bias(p, b, h, i, kj, n_kt64, &slot);
      const float prob = q_ok ? expf(s - lse_s[lane]) : 0.f;
      pv[r] = prob;
      dsv[r] = prob * (dpv[r] - dlt_s[lane]);
    }
    // dV += P^T dO, dK += dS^T Q: the warp's P and dS rows go through shared
    // tiles read four queries at a time (broadcast), each dO / Q value is read
    // once for the warp's keys
    float* p_w = p_tile + warp * kRowsPerWarp * kChunk;
    float* ds_w = ds_tile + warp * kRowsPerWarp * kChunk;
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      p_w[r * kChunk + lane] = pv[r];
      ds_w[r * kChunk + lane] = dsv[r];
    }
    __syncwarp();
    for (int j0 = 0; j0 < kChunk; j0 += 4) {
      float4 p4[kRowsPerWarp], d4[kRowsPerWarp];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        p4[r] = *reinterpret_cast<const float4*>(p_w + r * kChunk + j0);
        d4[r] = *reinterpret_cast<const float4*>(ds_w + r * kChunk + j0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float gv[TD], qv[TD];
#pragma unroll
        for (int t = 0; t < TD; ++t) {
          const int d = lane + 32 * t;
          gv[t] = d < D ? go_s[(j0 + u) * Dp + d] : 0.f;
          qv[t] = d < D ? q_s[(j0 + u) * Dp + d] : 0.f;
        }
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
          const float pj = u == 0 ? p4[r].x : u == 1 ? p4[r].y : u == 2 ? p4[r].z : p4[r].w;
          const float dsj = u == 0 ? d4[r].x : u == 1 ? d4[r].y : u == 2 ? d4[r].z : d4[r].w;
#pragma unroll
          for (int t = 0; t < TD; ++t) {
            dv[r][t] = fmaf(pj, gv[t], dv[r][t]);
            dk[r][t] = fmaf(dsj, qv[t], dk[r][t]);
          }
        }
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int64_t kj = key0 + warp * kRowsPerWarp + r;
    if (kj >= N) continue;
#pragma unroll
    for (int t = 0; t < TD; ++t) {
      const int d = lane + 32 * t;
      if (d >= D) continue;
      const int64_t o = (((b * p.heads + h) * N) + kj) * D + d;
      if (bp.grad_k != nullptr) bp.grad_k[o] = dk[r][t] * p.scale;
      if (bp.grad_v != nullptr) bp.grad_v[o] = dv[r][t];
    }
  }
}

// C[a,f] = -sum_c G[a,c] * sign(X[a,f] - Y[c,f]); G[a,c] at a * g_a + c * g_c.
// CTA: 64 a x 64 f, 256 threads with 4 x 4 outputs each; c streamed in chunks of 16.
constexpr int kNA = 64, kNF = 64, kNC = 16;
__global__ void __launch_bounds__(256) nl1_sign_kernel(const float* __restrict__ X, const float* __restrict__ Y,
                                                       const float* __restrict__ G, int64_t g_a, int64_t g_c,
                                                       float* __restrict__ C, int64_t A, int64_t Cn, int64_t F) {
  __shared__ float y_s[kNC][kNF + 1];
  __shared__ float g_s[kNC][kNA + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // f micro-tile tx, a micro-tile ty
  const int64_t a0 = static_cast<int64_t>(blockIdx.y) * kNA, f0 = static_cast<int64_t>(blockIdx.x) * kNF;
  float x[4][4], acc[4][4];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int64_t a = a0 + ty + 16 * u, f = f0 + tx + 16 * v;
      x[u][v] = (a < A && f < F) ? X[a * F + f] : 0.f;
      acc[u][v] = 0.f;
    }
  for (int64_t c0 = 0; c0 < Cn; c0 += kNC) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < kNC * kNF; idx += 256) {
      const int c = idx / kNF, f = idx % kNF;
      y_s[c][f] = (c0 + c < Cn && f0 + f < F) ? Y[(c0 + c) * F + f0 + f] : 0.f;
    }
    for (int idx = threadIdx.x; idx < kNC * kNA; idx += 256) {
      const int c = idx / kNA, a = idx % kNA;
      g_s[c][a] = (c0 + c < Cn && a0 + a < A) ? G[(a0 + a) * g_a + (c0 + c) * g_c] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < kNC; ++c) {
      float yv[4], gv[4];
#pragma unroll
      for (int v = 0; v < 4; ++v) yv[v] = y_s[c][tx + 16 * v];
#pragma unroll
      for (int u = 0; u < 4; ++u) gv[u] = g_s[c][ty + 16 * u];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float d = x[u][v] - yv[v];
          // g * sign(d): flip g's sign bit when d < 0; zero when d == 0
          const float t = __uint_as_float(__float_as_uint(gv[u]) ^ (__float_as_uint(d) & 0x80000000u));
          acc[u][v] += d != 0.f ? t : 0.f;
        }
    }
  }
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int64_t a = a0 + ty + 16 * u, f = f0 + tx + 16 * v;
      if (a < A && f < F) C[a * F + f] = -acc[u][v];
    }
}

}  // namespace

int32_t launch_sla_backward(const SlaBwdParams& bp, cudaStream_t stream) {
  const SlaParams& p = bp.f;
  if (p.head_dim < 1 || p.head_dim > kMaxDim) return 8;
  if (p.bias_mode != 0 && p.poses > kMaxBwdPoses) return 8;
  if (p.heads > 65535 || p.batch > 65535) return 8;
  const int64_t rows = p.batch * p.heads * p.seq;
  delta_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(bp);
  const int Dp = row_stride(static_cast<int>(p.head_dim));
  const int P = p.bias_mode != 0 ? static_cast<int>(p.poses) : 0;
  const size_t smem_rows =
      (static_cast<size_t>(2 * kRows + 2 * kChunk) * Dp + kRows * kChunk + kRows * P) * sizeof(float);
  const size_t smem_cols =
      (static_cast<size_t>(2 * kRows + 2 * kChunk) * Dp + 2 * kRows * kChunk + 2 * kChunk) * sizeof(float);
  const int td = p.head_dim <= 32 ? 1 : p.head_dim <= 64 ? 2 : 4;
  auto rows_k = td == 1 ? rows_kernel<1> : td == 2 ? rows_kernel<2> : rows_kernel<4>;
  auto cols_k = td == 1 ? cols_kernel<1> : td == 2 ? cols_kernel<2> : cols_kernel<4>;
  if (smem_rows > 48 * 1024 &&
      cudaFuncSetAttribute(rows_k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_rows)) !=
          cudaSuccess)
    return 6;
  if (smem_cols > 48 * 1024 &&
      cudaFuncSetAttribute(cols_k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_cols)) !=
          cudaSuccess)
    return 6;
  const dim3 grid(static_cast<unsigned>((p.seq + kRows - 1) / kRows), static_cast<unsigned>(p.heads),
                  static_cast<unsigned>(p.batch));
  if (bp.grad_q || bp.grad_pose || bp.grad_fields || bp.grad_dense)
    rows_k<<<grid, kWarps * 32, smem_rows, stream>>>(bp);
  if (bp.grad_k || bp.grad_v) cols_k<<<grid, kWarps * 32, smem_cols, stream>>>(bp);
  return cudaGetLastError() == cudaSuccess ? 0 : 6;
}

int32_t launch_nl1_backward(const float* x, const float* w, const float* grad_out, float* grad_x, float* grad_w,
                            int64_t rows, int64_t protos, int64_t features, cudaStream_t stream) {
  if (grad_x != nullptr) {
    const dim3 grid(static_cast<unsigned>((features + kNF - 1) / kNF), static_cast<unsigned>((rows + kNA - 1) / kNA));
    if (grid.y > 65535u) return 8;
    // grad_x[m,f] = -sum_p g[m,p] sign(x[m,f] - w[p,f])
    nl1_sign_kernel<<<grid, 256, 0, stream>>>(x, w, grad_out, protos, 1, grad_x, rows, protos, features);
  }
  if (grad_w != nullptr) {
    const dim3 grid(static_cast<unsigned>((features + kNF - 1) / kNF), static_cast<unsigned>((protos + kNA - 1) / kNA));
    if (grid.y > 65535u) return 8;
    // grad_w[p,f] = sum_m g[m,p] sign(x[m,f] - w[p,f]) = -sum_m g[m,p] sign(w[p,f] - x[m,f])
    nl1_sign_kernel<<<grid, 256, 0, stream>>>(w, x, grad_out, 1, protos, grad_w, protos, rows, features);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 6;
}

}  // namespace intp
