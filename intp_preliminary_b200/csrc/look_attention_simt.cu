// look_attention_simt.cu - CUDA-core structured Look attention forward.
//
// This is the coverage path: every dtype (f32/f16/bf16), any head_dim <= 128,
// any strides, every bias mode (none / general fields / slots / slot fields) and the
// optional dense bias.  It computes exactly the reference semantics
// (layers/triton_structured_look_attention.py:25-54):
//   S = scale * q k^T (fp32);  S[1:,1:] += sum_p pose * fields  (+ dense);
//   O = softmax(S) v,  LSE = logsumexp(S)
// with fp32 accumulation everywhere, so it is also the fp32 parity path.
//
// Layout: one CTA = 4 warps = 16 query rows of one (batch, head); the key axis
// is streamed in chunks of 32 keys staged in shared memory as fp32; lane j of a
// warp owns key j of the chunk for the logits and output dims lane+32i for the
// accumulator.  Online (flash) softmax per row.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "sla_internal.h"

namespace intp {
namespace {

constexpr int kRows = 16;      // query rows per CTA
constexpr int kWarps = 4;
constexpr int kRowsPerWarp = kRows / kWarps;
constexpr int kKeys = 32;      // keys per chunk
constexpr int kMaxDim = 128;

__device__ __forceinline__ float load_any(const void* p, int64_t idx, int32_t dtype) {
  switch (dtype) {
    case 1: return __half2float(static_cast<const __half*>(p)[idx]);
    case 2: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
    default: return static_cast<const float*>(p)[idx];
  }
}

__device__ __forceinline__ void store_any(void* p, int64_t idx, int32_t dtype, float v) {
  switch (dtype) {
    case 1: static_cast<__half*>(p)[idx] = __float2half_rn(v); break;
    case 2: static_cast<__nv_bfloat16*>(p)[idx] = __float2bfloat16_rn(v); break;
    default: static_cast<float*>(p)[idx] = v; break;
  }
}

__global__ void __launch_bounds__(kWarps * 32)
sla_simt_kernel(const SlaParams p) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t b = blockIdx.z;
  const int64_t h = blockIdx.y;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int64_t N = p.seq;
  const int D = static_cast<int>(p.head_dim);
  const int Dp = D + 1;  // padded smem row stride (bank-conflict free)

  extern __shared__ float smem[];
  float* q_s = smem;                      // kRows x Dp
  float* k_s = q_s + kRows * Dp;          // kKeys x Dp
  float* v_s = k_s + kKeys * Dp;          // kKeys x Dp

  // Stage the CTA's query rows.
  for (int idx = threadIdx.x; idx < kRows * D; idx += blockDim.x) {
    const int r = idx / D, d = idx % D;
    const int64_t i = row0 + r;
    float val = 0.f;
    if (i < N) val = load_any(p.q, b * p.q_stride[0] + h * p.q_stride[1] + i * p.q_stride[2] + d, p.dtype);
    q_s[r * Dp + d] = val;
  }

  float m[kRowsPerWarp], l[kRowsPerWarp], acc[kRowsPerWarp][kMaxDim / 32];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int t = 0; t < kMaxDim / 32; ++t) acc[r][t] = 0.f;
  }

  const int64_t patch_count = N - 1;
  const int64_t n_kt64 = (N + 63) / 64;

  for (int64_t key0 = 0; key0 < N; key0 += kKeys) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < kKeys * D; idx += blockDim.x) {
      const int j = idx / D, d = idx % D;
      const int64_t kj = key0 + j;
      float kv = 0.f, vv = 0.f;
      if (kj < N) {
        kv = load_any(p.k, b * p.k_stride[0] + h * p.k_stride[1] + kj * p.k_stride[2] + d, p.dtype);
        vv = load_any(p.v, b * p.v_stride[0] + h * p.v_stride[1] + kj * p.v_stride[2] + d, p.dtype);
      }
      k_s[j * Dp + d] = kv;
      v_s[j * Dp + d] = vv;
    }
    __syncthreads();

    const int64_t kj = key0 + lane;
    const bool key_ok = kj < N;
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int rr = warp * kRowsPerWarp + r;
      const int64_t i = row0 + rr;
      if (i >= N) continue;  // warp-uniform
      float s = 0.f;
      for (int d = 0; d < D; ++d) s = fmaf(q_s[rr * Dp + d], k_s[lane * Dp + d], s);
      s *= p.scale;
      if (key_ok && i > 0 && kj > 0) {
        const int64_t pq = i - 1, pk = kj - 1;
        float bias = 0.f;
        if (p.bias_mode == 1) {
          for (int64_t pp = 0; pp < p.poses; ++pp) {
            const float w = load_any(p.pose, b * p.pose_stride[0] + pq * p.pose_stride[1] +
                                                 h * p.pose_stride[2] + pp * p.pose_stride[3],
                                     p.pose_dtype);
            const float f = load_any(p.fields, h * p.fields_stride[0] + pp * p.fields_stride[1] +
                                                   pq * p.fields_stride[2] + pk * p.fields_stride[3],
                                     p.fields_dtype);
            bias = fmaf(w, f, bias);
          }
        } else if (p.bias_mode == 2) {
          const int64_t qt = i >> 7, kt = kj >> 6;
          const int64_t off = (qt * n_kt64 + kt) * 8192 + ((kj & 63) >> 4) * 2048 + (i & 127) * 16 + (kj & 15);
          const int slot = p.slots_packed[off];
          if (slot < p.poses)
            bias = load_any(p.pose, b * p.pose_stride[0] + pq * p.pose_stride[1] + h * p.pose_stride[2] +
                                        slot * p.pose_stride[3],
                            p.pose_dtype);
        } else if (p.bias_mode == 3) {
          const int64_t qt = i >> 7, kt = kj >> 6;
          const int64_t off = (qt * n_kt64 + kt) * 8192 + ((kj & 63) >> 4) * 2048 + (i & 127) * 16 + (kj & 15);
          const int slot = p.slots_packed[off];
          if (slot < p.slots) {
            for (int64_t pp = 0; pp < p.poses; ++pp) {
              const float w = load_any(p.pose, b * p.pose_stride[0] + pq * p.pose_stride[1] +
                                                   h * p.pose_stride[2] + pp * p.pose_stride[3],
                                       p.pose_dtype);
              const float f = load_any(p.fields, h * p.fields_stride[0] + pp * p.fields_stride[1] +
                                                     slot * p.fields_stride[2],
                                       p.fields_dtype);
              bias = fmaf(w, f, bias);
            }
          }
        }
        if (p.dense != nullptr)
          bias += load_any(p.dense, b * p.dense_stride[0] + h * p.dense_stride[1] + pq * p.dense_stride[2] +
                                        pk * p.dense_stride[3],
                           p.dense_dtype);
        s += bias;
      }
      if (!key_ok) s = -INFINITY;
      float cmax = s;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
      const float m_new = fmaxf(m[r], cmax);
      const float alpha = expf(m[r] - m_new);  // exp(-inf) = 0 on the first chunk
      const float e = key_ok ? expf(s - m_new) : 0.f;
      float csum = e;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) csum += __shfl_xor_sync(0xffffffffu, csum, o);
      l[r] = l[r] * alpha + csum;
      m[r] = m_new;
#pragma unroll
      for (int t = 0; t < kMaxDim / 32; ++t) acc[r][t] *= alpha;
      for (int j = 0; j < kKeys; ++j) {
        const float pj = __shfl_sync(0xffffffffu, e, j);
#pragma unroll
        for (int t = 0; t < kMaxDim / 32; ++t) {
          const int d = lane + 32 * t;
          if (d < D) acc[r][t] = fmaf(pj, v_s[j * Dp + d], acc[r][t]);
        }
      }
      (void)patch_count;
    }
  }

#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int64_t i = row0 + warp * kRowsPerWarp + r;
    if (i >= N) continue;
    const float inv = 1.f / l[r];
#pragma unroll
    for (int t = 0; t < kMaxDim / 32; ++t) {
      const int d = lane + 32 * t;
      if (d < D)
        store_any(p.out, b * p.out_stride[0] + h * p.out_stride[1] + i * p.out_stride[2] + d, p.dtype,
                  acc[r][t] * inv);
    }
    if (p.lse != nullptr && lane == 0) p.lse[(b * p.heads + h) * N + i] = m[r] + logf(l[r]);
  }
}

}  // namespace

int32_t launch_sla_simt(const SlaParams& p, cudaStream_t stream) {
  if (p.head_dim < 1 || p.head_dim > kMaxDim) return 8;  // INTP_ERR_UNSUPPORTED
  const int Dp = static_cast<int>(p.head_dim) + 1;
  const size_t smem = static_cast<size_t>(kRows + 2 * kKeys) * Dp * sizeof(float);
  dim3 grid(static_cast<unsigned>((p.seq + kRows - 1) / kRows), static_cast<unsigned>(p.heads),
            static_cast<unsigned>(p.batch));
  if (grid.y > 65535u || grid.z > 65535u) return 8;
  sla_simt_kernel<<<grid, kWarps * 32, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : 6;
}

}  // namespace intp
