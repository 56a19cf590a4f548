// backward_tc.cu - tensor-core half of the structured-Look-attention backward
// (sm_100a, bf16 / f16, head_dim 64, SLOTS or no Look bias).
//
// The reference's backward (layers/triton_structured_look_attention.py:341-409)
// materialises the probabilities P and the logit gradient dS as B*H*N*N
// tensors (its Triton pass :172-292) and then runs batched matmuls.  This
// kernel produces the same two tensors on the tensor cores, in 16-bit, plus
// the Look (slot) gradient; the caller finishes with three batched GEMMs
// (dV = P^T dO, dK = dS^T Q, dQ = dS K).  Per 128-query tile and 64-key tile:
//   S  = Q K^T      and  dP = dO V^T      (tcgen05.mma, both into TMEM)
//   P  = exp(scale S + bias - lse)        (bias from the SLOTS table, log2 domain)
//   dS = P (dP - delta),  delta = rowsum(dO * O)
//   dpose[slot] += dS   (per query row, over the keys of that slot)
// and writes P and dS in the input dtype (the reference's `probability` and
// `score_grad`); the caller applies the softmax scale in the dQ / dK GEMMs.
//
// CTA: 288 threads, one (batch, head, 128-query tile) per CTA.  Warps 0-7 are
// two warpgroups of row threads: thread t owns query row t % 128 (its TMEM
// lane) and keys 0-31 (t < 128) or 32-63 of every key tile.  Warp 8 lane 0
// issues the TMA loads (Q, dO once; K / V tiles through a 2-stage ring) and the
// MMAs (S and dP into one of two TMEM buffers).  Each row thread reads its 32
// slot bytes of a tile straight from the packed pair table (L2) while it waits
// for the tile's scores; each warpgroup keeps its per-slot gradient sums in
// its own shared [slot][row] array (one writer per cell), added at the end.
// Every mbarrier wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "../../include/intp_b200.h"
#include "sla_internal.h"
#include "sla_look_table.cuh"
#include "sla_tc_common.cuh"
#include "sm100_ptx.cuh"

namespace intp {
namespace {

constexpr int BQ = 128;                     // query rows per tile
constexpr int BK = 64;                      // keys per tile
constexpr int D64 = 64;
constexpr int kRowThreads = 256;          // two warpgroups: keys 0-31 / 32-63 of each tile
constexpr int kBwdThreads = kRowThreads + 32;
constexpr int kMmaWarp = kRowThreads / 32;
constexpr uint32_t kTile128 = BQ * D64 * 2;  // 16 KB
constexpr uint32_t kTile64 = BK * D64 * 2;   // 8 KB

struct alignas(8) BwdBars {
  uint64_t qdo_full;
  uint64_t kv_full[2], kv_empty[2];
  uint64_t s_full[2], s_free[2];
  uint64_t drain;
  uint32_t tmem_base;
  int32_t abort;
};

struct BwdTcArgs {
  SlaParams p;
  MapOrder oq, odo, ok, ov;
  const void* dout;
  int64_t dout_stride[4];
  void* p_out;
  void* ds_out;
  int64_t ld;
  float* grad_pose;
  int32_t n_qt, n_kt, n_slots, pose_vec4;
  uint32_t off_table, off_dacc, off_bars;
  uint64_t wait_ns;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pk2(float lo, float hi) {
  return BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

// Barrier of the row threads only (named barrier 1).
__device__ __forceinline__ void row_threads_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kRowThreads) : "memory"); }

template <bool BF16>
__device__ __forceinline__ float ld16(const void* p, int64_t idx) {
  return BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx])
              : __half2float(static_cast<const __half*>(p)[idx]);
}

template <bool BF16>
__global__ void __launch_bounds__(kBwdThreads)
sla_bwd_pds_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                   const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                   const BwdTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* q_s = smem;
  uint8_t* do_s = smem + kTile128;
  uint8_t* k_s = smem + 2 * kTile128;            // 2 stages
  uint8_t* v_s = k_s + 2 * kTile64;              // 2 stages
  float* table_s = reinterpret_cast<float*>(smem + a.off_table);
  float* dacc_s = reinterpret_cast<float*>(smem + a.off_dacc);
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + a.off_bars);
  const SlaParams& p = a.p;
  volatile int32_t* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t H = static_cast<uint32_t>(p.heads);
  const int32_t N = static_cast<int32_t>(p.seq);
  const uint32_t item = blockIdx.x;
  const int32_t qt = static_cast<int32_t>(item % a.n_qt);
  const uint32_t bh = item / a.n_qt;
  const int32_t h = static_cast<int32_t>(bh % H), b = static_cast<int32_t>(bh / H);
  const bool use_bias = a.n_slots > 0;
  const int n_kt = a.n_kt;

  if (threadIdx.x == 0) {
    mbar_init(&bars->qdo_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_free[s], kRowThreads / 32);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    mbar_fence_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&bars->tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kMmaWarp) {
    // ------------------------------------------------------------ loads + MMAs (one thread)
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_do);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const int32_t r0 = qt * BQ;
      mbar_arrive_expect_tx(&bars->qdo_full, 2 * kTile128);
      tma_load_4d(q_s, &tm_q, &bars->qdo_full, 0, map_coord(a.oq, 1, r0, h, b), map_coord(a.oq, 2, r0, h, b),
                  map_coord(a.oq, 3, r0, h, b));
      tma_load_4d(do_s, &tm_do, &bars->qdo_full, 0, map_coord(a.odo, 1, r0, h, b), map_coord(a.odo, 2, r0, h, b),
                  map_coord(a.odo, 3, r0, h, b));
      auto load_kv = [&](int j) {
        const int st = j & 1;
        const int32_t r = j * BK;
        mbar_arrive_expect_tx(&bars->kv_full[st], 2 * kTile64);
        tma_load_4d(k_s + st * kTile64, &tm_k, &bars->kv_full[st], 0, map_coord(a.ok, 1, r, h, b),
                    map_coord(a.ok, 2, r, h, b), map_coord(a.ok, 3, r, h, b));
        tma_load_4d(v_s + st * kTile64, &tm_v, &bars->kv_full[st], 0, map_coord(a.ov, 1, r, h, b),
                    map_coord(a.ov, 2, r, h, b), map_coord(a.ov, 3, r, h, b));
      };
      const uint32_t idesc = idesc_f16(BF16, false, BQ, BK);
      const uint64_t q_desc = smem_desc_sw128(smem_u32(q_s), 16, 1024);
      const uint64_t do_desc = smem_desc_sw128(smem_u32(do_s), 16, 1024);
      int loaded = 0;
      bool ok = true, issued = false;
      load_kv(0);
      loaded = 1;
      ok = mbar_wait(&bars->qdo_full, 0, abort_flag, p.status, kDevTimeoutMma, a.wait_ns);
      for (int j = 0; j < n_kt && ok; ++j) {
        const int st = j & 1;
        if (j + 1 < n_kt) {
          // stage (j+1)&1 last held tile j-1: its MMAs committed kv_empty
          if (j + 1 >= 2 &&
              !mbar_wait(&bars->kv_empty[(j + 1) & 1], ((j - 1) >> 1) & 1, abort_flag, p.status, kDevTimeoutProducer,
                         a.wait_ns)) {
            ok = false;
            break;
          }
          load_kv(j + 1);
          loaded = j + 2;
        }
        if (!mbar_wait(&bars->kv_full[st], (j >> 1) & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) {
          ok = false;
          break;
        }
        // TMEM buffer st last held tile j-2: the softmax warps loaded it
        if (j >= 2 && !mbar_wait(&bars->s_free[st], ((j - 2) >> 1) & 1, abort_flag, p.status, kDevTimeoutMma,
                                 a.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t k_desc = smem_desc_sw128(smem_u32(k_s + st * kTile64), 16, 1024);
        const uint64_t v_desc = smem_desc_sw128(smem_u32(v_s + st * kTile64), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D64 / 16; ++kk)
          mma_ss(tmem + st * 128, q_desc + ((kk * 32) >> 4), k_desc + ((kk * 32) >> 4), idesc, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < D64 / 16; ++kk)
          mma_ss(tmem + st * 128 + 64, do_desc + ((kk * 32) >> 4), v_desc + ((kk * 32) >> 4), idesc,
                 kk > 0 ? 1u : 0u);
        mma_commit(&bars->s_full[st]);
        mma_commit(&bars->kv_empty[st]);
        issued = true;
      }
      volatile int32_t no_abort = 0;
      if (issued) {
        mma_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, &no_abort, p.status, kDevTimeoutDrain);
      }
      // Drain: every issued copy has landed before the CTA exits.
      mbar_wait(&bars->qdo_full, 0, &no_abort, p.status, kDevTimeoutDrain);
      for (int st = 0; st < 2; ++st) {
        const int cnt = loaded > st ? (loaded - st + 1) / 2 : 0;
        if (cnt > 0) mbar_wait(&bars->kv_full[st], (cnt - 1) & 1, &no_abort, p.status, kDevTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ row threads
    const int row = threadIdx.x & (BQ - 1);         // 0..127 = TMEM lane
    const int half = threadIdx.x >> 7;              // this thread's 32 keys of each tile
    const int32_t i = qt * BQ + row;                // query token
    const bool valid = i < N;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + 32 * half;
    const float scale_log2 = p.scale * kLog2eF;
    // delta = rowsum(dO * O) and the row's LSE (log2 domain)
    float delta = 0.f, lse2 = 0.f;
    if (valid) {
      const int64_t ob = b * p.out_stride[0] + h * p.out_stride[1] + int64_t(i) * p.out_stride[2];
      const int64_t gb = b * a.dout_stride[0] + h * a.dout_stride[1] + int64_t(i) * a.dout_stride[2];
#pragma unroll 8
      for (int d = 0; d < D64; ++d) delta = fmaf(ld16<BF16>(p.out, ob + d), ld16<BF16>(a.dout, gb + d), delta);
      lse2 = p.lse[(int64_t(b) * H + h) * N + i] * kLog2eF;
    }
    float* trow = table_s + row;
    // one slot-sum array per warpgroup: each cell has one writer (this thread)
    float* drow = dacc_s + half * (a.n_slots + 2) * BQ + row;
    if (use_bias) {
      if (half == 0) stage_table(table_s, a, b, h, i, row);  // log2-domain Look values; [ns] = 0, [ns+1] = -inf
      for (int s = 0; s < a.n_slots + 2; ++s) drow[s * BQ] = 0.f;
      row_threads_sync();
    }
    const uint8_t* sbase = p.slots_packed + int64_t(qt) * n_kt * kSlotTileBytes + row * 16;
    const int64_t orow = (int64_t(bh) * N + i) * a.ld;  // element offset of this row in P / dS
    bool ok = true;
    for (int j = 0; j < n_kt && ok; ++j) {
      const int st = j & 1;
      // this row's 64 slot bytes of the tile (L2), in flight during the wait
      uint4 cur[2];
      if (use_bias) {
        const uint8_t* src = sbase + int64_t(j) * kSlotTileBytes + half * 4096;
#pragma unroll
        for (int c = 0; c < 2; ++c) cur[c] = __ldg(reinterpret_cast<const uint4*>(src + c * 2048));
      }
      if (!mbar_wait(&bars->s_full[st], (j >> 1) & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[32], dr[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld16(lane_base + st * 128 + c * 16, *reinterpret_cast<uint32_t(*)[16]>(sr + 16 * c));
        tmem_ld16(lane_base + st * 128 + 64 + c * 16, *reinterpret_cast<uint32_t(*)[16]>(dr + 16 * c));
      }
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        reg_fence16(*reinterpret_cast<uint32_t(*)[16]>(sr + 16 * c));
        reg_fence16(*reinterpret_cast<uint32_t(*)[16]>(dr + 16 * c));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s_free[st]);  // the MMA may overwrite buffer st
      const int32_t k0 = j * BK + 32 * half;
      uint8_t* pdst = static_cast<uint8_t*>(a.p_out) + 2 * (orow + k0);
      uint8_t* ddst = static_cast<uint8_t*>(a.ds_out) + 2 * (orow + k0);
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 8 keys: one 16-byte store of P and of dS
        uint32_t pw[4], dw[4];
        if (use_bias) {
          // all eight table reads first, then the math, then the eight slot-sum updates
          uint32_t sl[8];
          float tb[8], g[8];
#pragma unroll
          for (int e2 = 0; e2 < 8; ++e2) {
            const int e = 8 * c + e2;
            sl[e2] = __byte_perm((&cur[e >> 4].x)[(e & 15) >> 2], 0u, 0x4440u | (e & 3));
            tb[e2] = trow[sl[e2] * BQ];
          }
#pragma unroll
          for (int e2 = 0; e2 < 8; e2 += 2) {
            const int e = 8 * c + e2;
            const float p0 = fast_exp2(fmaf(__uint_as_float(sr[e]), scale_log2, tb[e2]) - lse2);
            const float p1 = fast_exp2(fmaf(__uint_as_float(sr[e + 1]), scale_log2, tb[e2 + 1]) - lse2);
            g[e2] = p0 * (__uint_as_float(dr[e]) - delta);
            g[e2 + 1] = p1 * (__uint_as_float(dr[e + 1]) - delta);
            pw[e2 / 2] = pk2<BF16>(p0, p1);
            dw[e2 / 2] = pk2<BF16>(g[e2], g[e2 + 1]);
          }
#pragma unroll
#pragma unroll
          for (int e2 = 0; e2 < 8; ++e2) drow[sl[e2] * BQ] += g[e2];  // [ns], [ns + 1]: sinks
        } else {
#pragma unroll
          for (int e2 = 0; e2 < 8; e2 += 2) {
            const int e = 8 * c + e2;
            const float t0 = k0 + e < N ? __uint_as_float(sr[e]) * scale_log2 : -INFINITY;
            const float t1 = k0 + e + 1 < N ? __uint_as_float(sr[e + 1]) * scale_log2 : -INFINITY;
            const float p0 = fast_exp2(t0 - lse2), p1 = fast_exp2(t1 - lse2);
            const float g0 = p0 * (__uint_as_float(dr[e]) - delta), g1 = p1 * (__uint_as_float(dr[e + 1]) - delta);
            pw[e2 / 2] = pk2<BF16>(p0, p1);
            dw[e2 / 2] = pk2<BF16>(g0, g1);
          }
        }
        if (valid && k0 + 8 * c < N) {
          reinterpret_cast<uint4*>(pdst)[c] = make_uint4(pw[0], pw[1], pw[2], pw[3]);
          reinterpret_cast<uint4*>(ddst)[c] = make_uint4(dw[0], dw[1], dw[2], dw[3]);
        }
      }
    }
    if (use_bias) row_threads_sync();  // both warpgroups' slot sums are in
    if (ok && use_bias && half == 0 && a.grad_pose != nullptr && valid && i >= 1) {
      const int64_t np = N - 1;
      float* dst = a.grad_pose + ((int64_t(b) * np + (i - 1)) * H + h) * a.n_slots;
      const float* other = drow + (a.n_slots + 2) * BQ;
      for (int s = 0; s < a.n_slots; ++s) dst[s] = drow[s * BQ] + other[s * BQ];
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

uint32_t align16(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

}  // namespace

int32_t launch_sla_probability_score_grad(const SlaParams& p, const void* dout, const int64_t* dout_stride, void* p_out,
                                void* ds_out, int64_t ld, float* grad_pose, cudaStream_t stream) {
  if (!tc_common_ok(p)) return 8;
  if (p.dense != nullptr || (p.bias_mode != 0 && p.bias_mode != 2)) return 8;
  if (p.bias_mode == 2 && (p.poses < 1 || p.poses > kMaxLookSlots || !p.slots_packed)) return 8;
  if (!p.lse || !dout || !p_out || !ds_out) return 1;
  if (ld < p.seq || ld % 8 || reinterpret_cast<uintptr_t>(p_out) % 16 || reinterpret_cast<uintptr_t>(ds_out) % 16)
    return 4;
  if (!tma_stride_ok(dout, dout_stride)) return 8;
  BwdTcArgs a;
  a.p = p;
  a.dout = dout;
  for (int d = 0; d < 4; ++d) a.dout_stride[d] = dout_stride[d];
  a.p_out = p_out;
  a.ds_out = ds_out;
  a.ld = ld;
  a.grad_pose = grad_pose;
  a.n_qt = static_cast<int32_t>((p.seq + BQ - 1) / BQ);
  a.n_kt = static_cast<int32_t>((p.seq + BK - 1) / BK);
  a.n_slots = p.bias_mode == 2 ? static_cast<int32_t>(p.poses) : 0;
  a.pose_vec4 = (p.bias_mode == 2 && p.pose_dtype == 0 && p.pose_stride[3] == 1 && a.n_slots % 4 == 0 &&
                 reinterpret_cast<uintptr_t>(p.pose) % 16 == 0 && p.pose_stride[0] % 4 == 0 &&
                 p.pose_stride[1] % 4 == 0 && p.pose_stride[2] % 4 == 0)
                    ? 1 : 0;
  a.wait_ns = tc_wait_budget_ns();
  SlaParams pd = p;  // dO has q's shape and dtype
  CUtensorMap mq, mdo, mk, mv;
  if (!make_map(&mq, &a.oq, p.q, p.q_stride, p, BQ) || !make_map(&mdo, &a.odo, dout, dout_stride, pd, BQ) ||
      !make_map(&mk, &a.ok, p.k, p.k_stride, p, BK) || !make_map(&mv, &a.ov, p.v, p.v_stride, p, BK))
    return 4;
  const uint32_t table_bytes = a.n_slots > 0 ? static_cast<uint32_t>((a.n_slots + 2) * BQ * 4) : 0u;
  uint32_t off = 2 * kTile128 + 4 * kTile64;
  a.off_table = off;
  off += table_bytes;
  a.off_dacc = off;
  off += 2 * table_bytes;
  a.off_bars = align16(off, 64);
  const size_t smem = a.off_bars + sizeof(BwdBars) + 1024;
  const int64_t grid = p.batch * p.heads * a.n_qt;
  if (grid > INT32_MAX) return 8;
  auto kernel = p.dtype == 2 ? sla_bwd_pds_kernel<true> : sla_bwd_pds_kernel<false>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return 6;
  kernel<<<static_cast<unsigned>(grid), kBwdThreads, smem, stream>>>(mq, mdo, mk, mv, a);
  return cudaGetLastError() == cudaSuccess ? 0 : 6;
}

}  // namespace intp
