// dense_look_grid.cu - bilinear sampling of per-query 4 x 12 Look grids into a
// dense (B, H, Q, K) attention bias, and its gradient with respect to the grids
// (C ABI dlg_forward / dlg_backward in include/intp_b200.h).
//
// The sampling tables (radial / angular corner indices, fractions, validity)
// depend on the (query, key) pair only, so one CTA takes one query and a chunk
// of (batch, head) rows: each key's four corners and bilinear weights are read
// once and reused for every row of the chunk.  Both kernels are bound by HBM
// traffic of the dense bias (written by the forward, read by the backward).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "../../include/intp_b200.h"

namespace intp {
namespace {

constexpr int kThreads = 256;
constexpr int kCells = 48;          // 4 radial x 12 angular grid cells
constexpr int kAngular = 12;
constexpr int kRadial = 4;
constexpr int kFwdRows = 64;        // (batch, head) rows per forward CTA
constexpr int kBwdRows = 128;       // (batch, head) rows per backward CTA
constexpr int kBwdSubRows = 32;     // rows of grad_output staged at a time
constexpr int kMaxKeysBwd = 1024;   // keys whose corner lists fit shared memory

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// The four corners of pair (q, k): grid cells r * 12 + a and their bilinear
// weights (1 - rw)(1 - aw), (1 - rw) aw, rw (1 - aw), rw aw, in the order
// (r0, a0), (r0, a1), (r1, a0), (r1, a1) of the reference's sampler
// (layers/triton_dense_look_grid.py:19-49, 89-108).  Pairs that are not valid,
// and corner indices outside the 4 x 12 grid, get weight 0 and cell 0.
struct Corners {
  int cell[4];
  float w[4];
};

__device__ __forceinline__ Corners pair_corners(const dlg_args& a, int64_t q, int64_t k) {
  Corners c;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    c.cell[j] = 0;
    c.w[j] = 0.f;
  }
  if (a.valid[q * a.table_stride[6][0] + k * a.table_stride[6][1]] == 0) return c;
  const int64_t r0 = a.radial0[q * a.table_stride[0][0] + k * a.table_stride[0][1]];
  const int64_t r1 = a.radial1[q * a.table_stride[1][0] + k * a.table_stride[1][1]];
  const int64_t a0 = a.angular0[q * a.table_stride[2][0] + k * a.table_stride[2][1]];
  const int64_t a1 = a.angular1[q * a.table_stride[3][0] + k * a.table_stride[3][1]];
  const float rw = a.radial_fraction[q * a.table_stride[4][0] + k * a.table_stride[4][1]];
  const float aw = a.angular_fraction[q * a.table_stride[5][0] + k * a.table_stride[5][1]];
  const int64_t rs[4] = {r0, r0, r1, r1};
  const int64_t as[4] = {a0, a1, a0, a1};
  const float ws[4] = {(1.f - rw) * (1.f - aw), (1.f - rw) * aw, rw * (1.f - aw), rw * aw};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (rs[j] >= 0 && rs[j] < kRadial && as[j] >= 0 && as[j] < kAngular) {
      c.cell[j] = static_cast<int>(rs[j] * kAngular + as[j]);
      c.w[j] = ws[j];
    }
  }
  return c;
}

// ---------------------------------------------------------------- forward
// CTA (q, row chunk): the chunk's grid rows (48 cells each, fp32) in shared
// memory, loaded kLoadBatch at a time per thread (independent loads in
// flight), with each row's (b, h) offsets worked out once; each thread takes
// keys k = tid, tid + 256, ... and writes out[b, h, q, k] for every row of the
// chunk (consecutive threads, consecutive keys: coalesced when the key stride
// is 1).  Four-key vector stores measured no faster (51 vs 49 us at B256 H3
// Q196): the kernel is not store-instruction bound.
constexpr int kLoadBatch = 12;

template <typename T>
__global__ void __launch_bounds__(kThreads) dlg_forward_kernel(const dlg_args a) {
  __shared__ float cells[kFwdRows][kCells];
  __shared__ int64_t out_row[kFwdRows];
  __shared__ int64_t grid_row[kFwdRows];
  const T* grid = static_cast<const T*>(a.grid);
  T* out = static_cast<T*>(a.out);
  const int64_t q = blockIdx.x;
  const int64_t rows = a.batch * a.heads;
  const int64_t bh0 = static_cast<int64_t>(blockIdx.y) * kFwdRows;
  const int nrows = static_cast<int>(min(static_cast<int64_t>(kFwdRows), rows - bh0));
  for (int rl = threadIdx.x; rl < nrows; rl += kThreads) {  // (b, h) of each row, once
    const int64_t bh = bh0 + rl, b = bh / a.heads, h = bh - b * a.heads;
    out_row[rl] = b * a.out_stride[0] + h * a.out_stride[1] + q * a.out_stride[2];
    grid_row[rl] = b * a.grid_stride[0] + q * a.grid_stride[1] + h * a.grid_stride[2];
  }
  __syncthreads();
  const int total = nrows * kCells;
  for (int i0 = threadIdx.x; i0 < total; i0 += kLoadBatch * kThreads) {
    float v[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = i0 + u * kThreads;
      v[u] = 0.f;
      if (i < total) {
        const int rl = i / kCells, c = i - rl * kCells;
        const int r = c / kAngular, an = c - r * kAngular;
        v[u] = to_f32(grid[grid_row[rl] + r * a.grid_stride[3] + an * a.grid_stride[4]]);
      }
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = i0 + u * kThreads;
      if (i < total) cells[i / kCells][i % kCells] = v[u];
    }
  }
  __syncthreads();
  for (int64_t k = threadIdx.x; k < a.queries; k += kThreads) {
    const Corners c = pair_corners(a, q, k);
    const int64_t ko = k * a.out_stride[3];
#pragma unroll 4
    for (int rl = 0; rl < nrows; ++rl) {
      const float* g = cells[rl];
      float v = g[c.cell[0]] * c.w[0];
      v = fmaf(g[c.cell[1]], c.w[1], v);
      v = fmaf(g[c.cell[2]], c.w[2], v);
      v = fmaf(g[c.cell[3]], c.w[3], v);
      out[out_row[rl] + ko] = from_f32<T>(v);
    }
  }
}

// ---------------------------------------------------------------- backward
// grad_grid[b, q, h, cell] = sum over keys k and corners j with cell_j(q, k) =
// cell of grad_out[b, h, q, k] * w_j(q, k)  (the reference's scatter_add,
// layers/triton_dense_look_grid.py:142-165).  For the CTA's query every key's
// corners are listed once per cell, in (key, corner) order, so each grid cell is
// a short sum in a fixed order (deterministic, fp32), then grad_out rows are
// staged kBwdSubRows at a time (kLoadBatch independent loads per thread in
// flight); a warp sums one cell for 32 rows at once (lane = row) into a
// shared tile that is written out coalesced.
template <typename T>
__global__ void __launch_bounds__(kThreads) dlg_backward_kernel(const dlg_args a, const void* __restrict__ grad_out,
                                                                 dlg_grad_strides gs, void* __restrict__ grad_grid) {
  extern __shared__ __align__(16) float smem_bwd[];
  const int K = static_cast<int>(a.queries);
  const int Kp = K | 1;                                     // odd row stride: lanes on rows hit distinct banks
  float* gsub = smem_bwd;                                   // [kBwdSubRows][Kp]
  float* out_s = gsub + kBwdSubRows * Kp;                   // [kBwdSubRows][kCells + 1]
  float* entry_w = out_s + kBwdSubRows * (kCells + 1);      // [4K]
  int* entry_k = reinterpret_cast<int*>(entry_w + 4 * K);   // [4K]
  uint32_t* key_cells = reinterpret_cast<uint32_t*>(entry_k + 4 * K);  // [K] four cells, a byte each (255: none)
  float* key_w = reinterpret_cast<float*>(key_cells + K);   // [K][4]
  __shared__ int seg_begin[kCells * 4 + 1];  // (cell, corner) segments, cell-major
  __shared__ int seg_fill[kCells * 4];
  __shared__ int64_t go_row[kBwdSubRows];
  __shared__ int64_t gg_row[kBwdSubRows];
  const T* go = static_cast<const T*>(grad_out);
  T* gg = static_cast<T*>(grad_grid);

  const int64_t q = blockIdx.x;
  const int64_t rows = a.batch * a.heads;
  const int64_t bh0 = static_cast<int64_t>(blockIdx.y) * kBwdRows;
  const int nrows = static_cast<int>(min(static_cast<int64_t>(kBwdRows), rows - bh0));

  for (int i = threadIdx.x; i < kCells * 4; i += kThreads) seg_fill[i] = 0;
  __syncthreads();
  for (int k = threadIdx.x; k < K; k += kThreads) {
    const Corners c = pair_corners(a, q, k);
    uint32_t packed = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool used = c.w[j] != 0.f;
      packed |= (used ? static_cast<uint32_t>(c.cell[j]) : 255u) << (8 * j);
      key_w[4 * k + j] = c.w[j];
      if (used) atomicAdd(&seg_fill[c.cell[j] * 4 + j], 1);  // counts only: order-independent
    }
    key_cells[k] = packed;
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // exclusive scan of the 192 segment sizes, 6 per lane
    const int lane = threadIdx.x;
    int local[6], sum = 0;
#pragma unroll
    for (int u = 0; u < 6; ++u) {
      local[u] = seg_fill[6 * lane + u];
      seg_fill[6 * lane + u] = 0;  // from here on: places already taken in the segment
      sum += local[u];
    }
    int incl = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += t;
    }
    int run = incl - sum;
#pragma unroll
    for (int u = 0; u < 6; ++u) {
      seg_begin[6 * lane + u] = run;
      run += local[u];
    }
    if (lane == 31) seg_begin[kCells * 4] = run;
  }
  __syncthreads();
  // Warp j lists corner j of every key, 32 keys at a time in key order; lanes
  // with the same cell take consecutive places (rank among equal cells).  Each
  // (cell, corner) segment is written by one warp only, so the order of every
  // cell's list is fixed: (corner, key).
  if (threadIdx.x < 4 * 32) {
    const int j = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int k0 = 0; k0 < K; k0 += 32) {
      const int k = k0 + lane;
      const uint32_t cell = k < K ? (key_cells[k] >> (8 * j)) & 0xffu : 255u;
      const uint32_t same = __match_any_sync(0xffffffffu, cell);
      const int rank = __popc(same & ((1u << lane) - 1u));
      const int seg = static_cast<int>(cell) * 4 + j;
      const int place = cell != 255u ? seg_begin[seg] + seg_fill[seg] + rank : 0;
      __syncwarp();
      if (cell != 255u) {
        entry_k[place] = k;
        entry_w[place] = key_w[4 * k + j];
        if (rank == 0) seg_fill[seg] += __popc(same);
      }
      __syncwarp();
    }
  }

  // element i of a sub-chunk is (row i / K, key i % K); a thread's elements
  // advance by kThreads, i.e. by step_r rows and step_k keys
  const int step_r = kThreads / K, step_k = kThreads % K;
  for (int r0 = 0; r0 < nrows; r0 += kBwdSubRows) {
    const int sub = min(kBwdSubRows, nrows - r0);
    __syncthreads();  // the lists are complete; the previous sub-chunk is consumed
    if (threadIdx.x < sub) {  // (b, h) of each row, once
      const int64_t bh = bh0 + r0 + threadIdx.x, b = bh / a.heads, h = bh - b * a.heads;
      go_row[threadIdx.x] = b * gs.stride[0] + h * gs.stride[1] + q * gs.stride[2];
      gg_row[threadIdx.x] = ((b * a.queries + q) * a.heads + h) * kCells;  // grad_grid: contiguous (B, Q, H, 4, 12)
    }
    __syncthreads();
    const int total = sub * K;
    int rl = threadIdx.x / K, k = threadIdx.x % K;
    for (int i0 = threadIdx.x; i0 < total; i0 += kLoadBatch * kThreads) {
      float v[kLoadBatch];
      int dst[kLoadBatch];
      int ru = rl, ku = k;
#pragma unroll
      for (int u = 0; u < kLoadBatch; ++u) {
        const bool in = i0 + u * kThreads < total;
        v[u] = in ? to_f32(go[go_row[ru] + ku * gs.stride[3]]) : 0.f;
        dst[u] = in ? ru * Kp + ku : -1;
        ru += step_r;
        ku += step_k;
        if (ku >= K) {
          ku -= K;
          ++ru;
        }
      }
#pragma unroll
      for (int u = 0; u < kLoadBatch; ++u)
        if (dst[u] >= 0) gsub[dst[u]] = v[u];
      rl = ru;
      k = ku;
    }
    __syncthreads();
    // lane = row of the sub-chunk, warp w = cells w, w + 8, ...: every lane of a
    // warp walks the same list (broadcast loads, no divergence)
    {
      const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
      const float* grow = gsub + lane * Kp;
      for (int cell = warp; cell < kCells; cell += kThreads / 32) {
        float s = 0.f;
        for (int e = seg_begin[4 * cell]; e < seg_begin[4 * cell + 4]; ++e) s = fmaf(grow[entry_k[e]], entry_w[e], s);
        out_s[lane * (kCells + 1) + cell] = s;
      }
    }
    __syncthreads();
    for (int o = threadIdx.x; o < sub * kCells; o += kThreads) {
      const int orl = o / kCells, cell = o - orl * kCells;
      gg[gg_row[orl] + cell] = from_f32<T>(out_s[orl * (kCells + 1) + cell]);
    }
  }
}

size_t backward_smem(int64_t keys) {
  return static_cast<size_t>(kBwdSubRows * (keys | 1) + kBwdSubRows * (kCells + 1) + 4 * keys + 4 * keys + keys +
                             4 * keys) * 4;
}

intp_status check_args(const dlg_args* a) {
  if (!a) return INTP_ERR_ARGUMENT;
  if (a->batch < 0 || a->queries < 0 || a->heads < 0) return INTP_ERR_ARGUMENT;
  if (a->dtype != INTP_F32 && a->dtype != INTP_F16 && a->dtype != INTP_BF16) return INTP_ERR_DTYPE;
  if (a->batch == 0 || a->queries == 0 || a->heads == 0) return INTP_OK;
  if (!a->radial0 || !a->radial1 || !a->angular0 || !a->angular1 || !a->radial_fraction ||
      !a->angular_fraction || !a->valid)
    return INTP_ERR_ARGUMENT;
  if (a->queries > INT32_MAX || (a->batch * a->heads + kFwdRows - 1) / kFwdRows > 65535) return INTP_ERR_UNSUPPORTED;
  return INTP_OK;
}

}  // namespace
}  // namespace intp

using namespace intp;

extern "C" INTP_API intp_status dlg_forward(const dlg_args* a, void* stream) {
  const intp_status st = check_args(a);
  if (st != INTP_OK || a->batch == 0 || a->queries == 0 || a->heads == 0) return st;
  if (!a->grid || !a->out) return INTP_ERR_ARGUMENT;
  const dim3 grid(static_cast<unsigned>(a->queries),
                  static_cast<unsigned>((a->batch * a->heads + kFwdRows - 1) / kFwdRows));
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->dtype == INTP_F32)
    dlg_forward_kernel<float><<<grid, kThreads, 0, s>>>(*a);
  else if (a->dtype == INTP_F16)
    dlg_forward_kernel<__half><<<grid, kThreads, 0, s>>>(*a);
  else
    dlg_forward_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(*a);
  return cudaGetLastError() == cudaSuccess ? INTP_OK : INTP_ERR_LAUNCH;
}

extern "C" INTP_API intp_status dlg_backward(const dlg_args* a, const void* grad_out, const dlg_grad_strides* gs,
                                             void* grad_grid, void* stream) {
  const intp_status st = check_args(a);
  if (st != INTP_OK || a->batch == 0 || a->queries == 0 || a->heads == 0) return st;
  if (!grad_out || !gs || !grad_grid) return INTP_ERR_ARGUMENT;
  if (a->queries > kMaxKeysBwd) return INTP_ERR_UNSUPPORTED;
  const size_t smem = backward_smem(a->queries);
  auto kernel = a->dtype == INTP_F32   ? dlg_backward_kernel<float>
                : a->dtype == INTP_F16 ? dlg_backward_kernel<__half>
                                       : dlg_backward_kernel<__nv_bfloat16>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return INTP_ERR_LAUNCH;
  const dim3 grid(static_cast<unsigned>(a->queries),
                  static_cast<unsigned>((a->batch * a->heads + kBwdRows - 1) / kBwdRows));
  kernel<<<grid, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(*a, grad_out, *gs, grad_grid);
  return cudaGetLastError() == cudaSuccess ? INTP_OK : INTP_ERR_LAUNCH;
}
