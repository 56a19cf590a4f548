// backward_fused.cu - the structured-Look-attention backward on the tensor
// cores without the B*H*N*N probability / score-gradient tensors (sm_100a,
// bf16 / f16, head_dim 64, SLOTS or no Look bias, no dense bias).
//
// The reference (layers/triton_structured_look_attention.py:341-409) writes P
// and dS = P (dO V^T - delta) to memory and then runs dQ = scale dS K,
// dK = scale dS^T Q, dV = P^T dO and the Look gradient as batched products.
// Here two kernels recompute the score tiles instead, each keeping its GEMM
// operands on chip:
//
//   sla_bwd_dq_kernel   (one CTA per batch, head and 128-query tile; loops over
//                        64-key tiles)
//       S = Q K^T, dP = dO V^T  -> TMEM;  dS = P (dP - delta)  (row threads)
//       dS (16-bit) back into TMEM;  dQ += dS K  (tcgen05, A operand in TMEM)
//       per-slot sums of dS -> grad_pose;  delta = rowsum(dO * O) -> global
//   sla_bwd_dkdv_kernel (one CTA per batch, head and 128-key tile; loops over
//                        64-query tiles)
//       S^T = K Q^T, dP^T = V dO^T  -> TMEM;  P^T, dS^T (row threads, one key
//       row each; the Look bias through the transposed slot table)
//       dV += P^T dO,  dK += dS^T Q  (tcgen05, A operands in TMEM)
//
// Both kernels: 288 threads.  Warps 0-7 are two warpgroups of row threads
// (thread t owns TMEM lane t % 128 and columns 0-31 (t < 128) or 32-63 of each
// tile); warp 8 lane 0 issues the TMA loads (3-stage ring for the streamed
// operand) and the MMAs.  Score buffers are double-buffered in TMEM; the
// 16-bit P / dS overwrite the first half of the fp32 columns their own thread
// has already read.  No atomics to global memory: every output element has one
// writer, so results are deterministic.  Every mbarrier wait is bounded; on a
// timeout the kernel drains its copies and MMAs, frees TMEM and records the
// status word.
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

constexpr int D64 = 64;
constexpr int kRows = 128;                    // TMEM lanes: query rows (dq) / key rows (dkdv)
constexpr int kCols = 64;                     // streamed tile: keys (dq) / queries (dkdv)
constexpr int kDqRowThreads = 256;          // dq: 2 warpgroups x 32 columns of each key tile
constexpr int kKvRowThreads = 512;          // dkdv: 4 warpgroups x 16 columns of each query tile
constexpr int kStages = 3;
constexpr uint32_t kTileRows = kRows * D64 * 2;  // 16 KB
constexpr uint32_t kTileCols = kCols * D64 * 2;  // 8 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColAcc0 = 256, kColAcc1 = 320;  // dQ | dK, dV
constexpr uint32_t kMinSmem = 120 * 1024;           // one CTA per SM (it holds all 512 TMEM columns)

constexpr int kStageBufs = 3;                 // dkdv: stage blocks (tile t in block t % 3)

struct alignas(8) FusedBars {
  uint64_t fixed_full;                        // the CTA's resident operand pair
  uint64_t stage_full[kStageBufs];            // dkdv: a stage block's copies landed (every row thread)
  uint64_t stage_free[kStageBufs];            // dkdv: every row warp has read a stage block
  uint64_t ring_full[kStages], ring_empty[kStages];
  uint64_t s_full[2], ready[2], buf_free[2];
  uint64_t acc_full, drain;
  uint32_t tmem_base;
  int32_t abort;
};

struct FusedArgs {
  SlaParams p;
  MapOrder o_fixed0, o_fixed1, o_ring0, o_ring1;  // dq: Q, dO | K, V;  dkdv: K, V | Q, dO
  const void* dout;
  int64_t dout_stride[4];
  float* grad_q;
  float* grad_k;
  float* grad_v;
  float* grad_pose;
  float* delta;
  const uint8_t* slots_t;                     // transposed packed slot table (dkdv)
  int32_t n_row_tiles, n_col_tiles, n_slots, pose_vec4, table_w;
  uint32_t off_table, off_dacc, off_bars;
  uint64_t wait_ns;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pk2(float lo, float hi) {
  return BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

// Barrier of the RT row threads only (named barrier 1).
template <int RT>
__device__ __forceinline__ void row_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(RT) : "memory");
}

// A 128-row x 64-column fp32 gradient block staged in shared memory for the
// epilogue: row r's 16-byte chunk c sits at chunk position c ^ (r & 15), so
// the row-per-thread float4 writes and the row-major float4 reads of the
// copy-out are both free of bank conflicts.  The copy-out moves whole
// consecutive rows, 32 float4 per warp instruction - where row-per-thread
// stores would touch 32 rows, a part of a sector each, per instruction.
__device__ __forceinline__ float4* blk_chunk(float* blk, int r, int c) {
  return reinterpret_cast<float4*>(blk + r * 64) + (c ^ (r & 15));
}
// Rows [0, rows) of a staged block to dst (64 floats per row, rows contiguous).
__device__ __forceinline__ void blk_copy_out(float* blk, float* dst, int rows, int tid, int nthreads) {
  for (int idx = tid; idx < rows * 16; idx += nthreads)
    reinterpret_cast<float4*>(dst)[idx] = *blk_chunk(blk, idx >> 4, idx & 15);
}

// Sum over 8 pairs of 16-bit values.
template <bool BF16>
__device__ __forceinline__ float dot8(uint4 x, uint4 y) {
  const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
  float acc = 0.f;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    float2 fx, fy;
    if (BF16) {
      fx = make_float2(__uint_as_float(xs[u] << 16), __uint_as_float(xs[u] & 0xffff0000u));
      fy = make_float2(__uint_as_float(ys[u] << 16), __uint_as_float(ys[u] & 0xffff0000u));
    } else {
      fx = __half22float2(*reinterpret_cast<const __half2*>(&xs[u]));
      fy = __half22float2(*reinterpret_cast<const __half2*>(&ys[u]));
    }
    acc = fmaf(fx.x, fy.x, acc);
    acc = fmaf(fx.y, fy.y, acc);
  }
  return acc;
}

// TMEM column of the 16-bit A operand for K-step kk (16 columns of the tile)
// when each warpgroup owns W consecutive columns and packs them (two per
// 32-bit column) into the first W / 2 of its own fp32 columns.
template <int W>
__device__ __forceinline__ uint32_t a_col(int kk) {
  return static_cast<uint32_t>((kk * 16 / W) * W + (kk * 16 % W) / 2);
}

// W (16 or 32) fp32 columns of S and of dP for this thread's lane.
template <int W>
__device__ __forceinline__ void load_scores(uint32_t taddr_s, uint32_t taddr_d, uint32_t (&sr)[W],
                                            uint32_t (&dr)[W]) {
#pragma unroll
  for (int c = 0; c < W / 16; ++c) {
    tmem_ld16(taddr_s + c * 16, *reinterpret_cast<uint32_t(*)[16]>(sr + 16 * c));
    tmem_ld16(taddr_d + c * 16, *reinterpret_cast<uint32_t(*)[16]>(dr + 16 * c));
  }
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < W / 16; ++c) {
    reg_fence16(*reinterpret_cast<uint32_t(*)[16]>(sr + 16 * c));
    reg_fence16(*reinterpret_cast<uint32_t(*)[16]>(dr + 16 * c));
  }
}

// Producer / MMA role shared by both kernels (warp 8, lane 0).  `fixed` is the
// pair loaded once (dq: Q, dO with 128 rows; dkdv: K, V), `ring` the pair
// streamed per tile (dq: K, V; dkdv: Q, dO with 64 rows).  Per tile t:
//   SCORE(t): X = F0 R0_t^T and Y = F1 R1_t^T into buffer t & 1
//   ACC(t):   dq:   acc0 += (16-bit TMEM X) R0_t
//             dkdv: acc1 += (TMEM X) R1_t,  acc0 += (TMEM Y) R0_t
// with SCORE(t + 1) issued before ACC(t) waits for the row threads.
template <bool BF16, bool KV, int W>
__device__ __forceinline__ void mma_role(const CUtensorMap* tm_f0, const CUtensorMap* tm_f1, const CUtensorMap* tm_r0,
                                         const CUtensorMap* tm_r1, const FusedArgs& a, FusedBars* bars,
                                         uint8_t* f0_s, uint8_t* f1_s, uint8_t* r0_s, uint8_t* r1_s, uint32_t tmem,
                                         int32_t row_tile, int32_t h, int32_t b) {
  const SlaParams& p = a.p;
  volatile int32_t* abort_flag = &bars->abort;
  tma_prefetch_desc(tm_f0);
  tma_prefetch_desc(tm_f1);
  tma_prefetch_desc(tm_r0);
  tma_prefetch_desc(tm_r1);
  const int32_t r0 = row_tile * kRows;
  mbar_arrive_expect_tx(&bars->fixed_full, 2 * kTileRows);
  tma_load_4d(f0_s, tm_f0, &bars->fixed_full, 0, map_coord(a.o_fixed0, 1, r0, h, b), map_coord(a.o_fixed0, 2, r0, h, b),
              map_coord(a.o_fixed0, 3, r0, h, b));
  tma_load_4d(f1_s, tm_f1, &bars->fixed_full, 0, map_coord(a.o_fixed1, 1, r0, h, b), map_coord(a.o_fixed1, 2, r0, h, b),
              map_coord(a.o_fixed1, 3, r0, h, b));
  const int n_t = a.n_col_tiles;
  auto load_ring = [&](int t) {
    const int s = t % kStages;
    const int32_t r = t * kCols;
    mbar_arrive_expect_tx(&bars->ring_full[s], 2 * kTileCols);
    tma_load_4d(r0_s + s * kTileCols, tm_r0, &bars->ring_full[s], 0, map_coord(a.o_ring0, 1, r, h, b),
                map_coord(a.o_ring0, 2, r, h, b), map_coord(a.o_ring0, 3, r, h, b));
    tma_load_4d(r1_s + s * kTileCols, tm_r1, &bars->ring_full[s], 0, map_coord(a.o_ring1, 1, r, h, b),
                map_coord(a.o_ring1, 2, r, h, b), map_coord(a.o_ring1, 3, r, h, b));
  };
  int loaded = 0;
  load_ring(0);
  loaded = 1;
  if (n_t > 1) {
    load_ring(1);
    loaded = 2;
  }
  const uint32_t idesc_s = idesc_f16(BF16, false, kRows, kCols);
  const uint32_t idesc_acc = idesc_f16(BF16, true, kRows, D64);
  const uint64_t f0_desc = smem_desc_sw128(smem_u32(f0_s), 16, 1024);
  const uint64_t f1_desc = smem_desc_sw128(smem_u32(f1_s), 16, 1024);
  bool ok = mbar_wait(&bars->fixed_full, 0, abort_flag, p.status, kDevTimeoutMma, a.wait_ns);
  bool issued = false;
  // ACC(t): wait for the row threads' 16-bit tile, then the accumulating MMAs.
  auto acc = [&](int t) -> bool {
    const int st = t & 1, s = t % kStages;
    if (!mbar_wait(&bars->ready[st], (t >> 1) & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) return false;
    tc_fence_after();
    // ring operands as MN-major B (K = the tile's 64 rows, N = head_dim)
    const uint64_t r0_desc = smem_desc_sw128(smem_u32(r0_s + s * kTileCols), kTileCols, 1024);
    const uint64_t r1_desc = smem_desc_sw128(smem_u32(r1_s + s * kTileCols), kTileCols, 1024);
    const uint32_t xb = tmem + st * 128, yb = xb + 64;
    if (KV) {
#pragma unroll
      for (int kk = 0; kk < kCols / 16; ++kk)  // dV += P^T dO
        mma_ts(tmem + kColAcc1, xb + a_col<W>(kk), r1_desc + ((kk * 2048) >> 4), idesc_acc, (t > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < kCols / 16; ++kk)  // dK += dS^T Q
        mma_ts(tmem + kColAcc0, yb + a_col<W>(kk), r0_desc + ((kk * 2048) >> 4), idesc_acc, (t > 0 || kk > 0) ? 1u : 0u);
    } else {
#pragma unroll
      for (int kk = 0; kk < kCols / 16; ++kk)  // dQ += dS K
        mma_ts(tmem + kColAcc0, xb + a_col<W>(kk), r0_desc + ((kk * 2048) >> 4), idesc_acc, (t > 0 || kk > 0) ? 1u : 0u);
    }
    mma_commit(&bars->buf_free[st]);
    mma_commit(&bars->ring_empty[s]);
    return true;
  };
  for (int t = 0; t < n_t && ok; ++t) {
    const int st = t & 1, s = t % kStages;
    // tile t + 1 goes to the stage of tile t - 2, free once ACC(t - 2) is done
    if (t >= 1 && t + 1 < n_t) {
      if (t >= 2 && !mbar_wait(&bars->ring_empty[(t + 1) % kStages], ((t - 2) / kStages) & 1, abort_flag, p.status,
                               kDevTimeoutProducer, a.wait_ns)) {
        ok = false;
        break;
      }
      load_ring(t + 1);
      loaded = t + 2;
    }
    if (!mbar_wait(&bars->ring_full[s], (t / kStages) & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) {
      ok = false;
      break;
    }
    if (t >= 2 &&
        !mbar_wait(&bars->buf_free[st], ((t - 2) >> 1) & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint64_t r0_desc = smem_desc_sw128(smem_u32(r0_s + s * kTileCols), 16, 1024);
    const uint64_t r1_desc = smem_desc_sw128(smem_u32(r1_s + s * kTileCols), 16, 1024);
#pragma unroll
    for (int kk = 0; kk < D64 / 16; ++kk)
      mma_ss(tmem + st * 128, f0_desc + ((kk * 32) >> 4), r0_desc + ((kk * 32) >> 4), idesc_s, kk > 0 ? 1u : 0u);
#pragma unroll
    for (int kk = 0; kk < D64 / 16; ++kk)
      mma_ss(tmem + st * 128 + 64, f1_desc + ((kk * 32) >> 4), r1_desc + ((kk * 32) >> 4), idesc_s,
             kk > 0 ? 1u : 0u);
    mma_commit(&bars->s_full[st]);
    issued = true;
    if (t >= 1 && !acc(t - 1)) {
      ok = false;
      break;
    }
  }
  if (ok && n_t > 0) {
    if (acc(n_t - 1))
      mma_commit(&bars->acc_full);
  }
  volatile int32_t no_abort = 0;
  if (issued) {
    mma_commit(&bars->drain);
    mbar_wait(&bars->drain, 0, &no_abort, p.status, kDevTimeoutDrain);
  }
  // every issued copy has landed before the CTA exits
  mbar_wait(&bars->fixed_full, 0, &no_abort, p.status, kDevTimeoutDrain);
  for (int s = 0; s < kStages; ++s) {
    const int cnt = loaded > s ? (loaded - s + kStages - 1) / kStages : 0;
    if (cnt > 0) mbar_wait(&bars->ring_full[s], (cnt - 1) & 1, &no_abort, p.status, kDevTimeoutDrain);
  }
}

__device__ __forceinline__ void init_bars(FusedBars* bars, uint32_t row_warps) {
  mbar_init(&bars->fixed_full, 1);
  for (int s = 0; s < kStages; ++s) {
    mbar_init(&bars->ring_full[s], 1);
    mbar_init(&bars->ring_empty[s], 1);
  }
  for (int s = 0; s < 2; ++s) {
    mbar_init(&bars->s_full[s], 1);
    mbar_init(&bars->ready[s], row_warps);
    mbar_init(&bars->buf_free[s], 1);
  }
  mbar_init(&bars->acc_full, 1);
  mbar_init(&bars->drain, 1);
  bars->abort = 0;
  mbar_fence_init();
}

// ============================================================================ dQ
constexpr int kDqThreads = kDqRowThreads + 32;
constexpr int kDqMmaWarp = kDqRowThreads / 32;

template <bool BF16>
__global__ void __launch_bounds__(kDqThreads, 1)
sla_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                  const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                  const FusedArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* q_s = smem;
  uint8_t* do_s = smem + kTileRows;
  uint8_t* k_s = smem + 2 * kTileRows;
  uint8_t* v_s = k_s + kStages * kTileCols;
  float* table_s = reinterpret_cast<float*>(smem + a.off_table);
  float* dacc_s = reinterpret_cast<float*>(smem + a.off_dacc);
  FusedBars* bars = reinterpret_cast<FusedBars*>(smem + a.off_bars);
  const SlaParams& p = a.p;
  volatile int32_t* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t H = static_cast<uint32_t>(p.heads);
  const int32_t N = static_cast<int32_t>(p.seq);
  const int32_t qt = static_cast<int32_t>(blockIdx.x % a.n_row_tiles);
  const uint32_t bh = blockIdx.x / a.n_row_tiles;
  const int32_t h = static_cast<int32_t>(bh % H), b = static_cast<int32_t>(bh / H);
  const bool use_bias = a.n_slots > 0;

  if (threadIdx.x == 0) init_bars(bars, kDqRowThreads / 32);
  if (warp == kDqMmaWarp) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kDqMmaWarp) {
    if (lane == 0) mma_role<BF16, false, 32>(&tm_q, &tm_do, &tm_k, &tm_v, a, bars, q_s, do_s, k_s, v_s, tmem, qt, h, b);
  } else {
    const int row = threadIdx.x & (kRows - 1);
    const int half = threadIdx.x >> 7;
    const int32_t i = qt * kRows + row;       // query token
    const bool valid = i < N;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float scale_log2 = p.scale * kLog2eF;
    float delta = 0.f, lse2 = 0.f;
    if (valid) {
      const uint4* o4 = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.out) +
                                                       2 * (b * p.out_stride[0] + h * p.out_stride[1] +
                                                            int64_t(i) * p.out_stride[2]));
      const uint4* g4 = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.dout) +
                                                       2 * (b * a.dout_stride[0] + h * a.dout_stride[1] +
                                                            int64_t(i) * a.dout_stride[2]));
      uint4 ov[8], gv[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        ov[c] = __ldg(o4 + c);
        gv[c] = __ldg(g4 + c);
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) delta += dot8<BF16>(ov[c], gv[c]);
      lse2 = p.lse[(int64_t(b) * H + h) * N + i] * kLog2eF;
      if (half == 0) a.delta[(int64_t(b) * H + h) * N + i] = delta;
    }
    float* trow = table_s + row;
    // one slot-sum array per warpgroup: every cell has a single writer, so the
    // sums are deterministic
    float* drow = dacc_s + half * (a.n_slots + 2) * kRows + row;
    if (use_bias) {
      if (half == 0) {
        stage_table(table_s, a, b, h, i, row);  // log2-domain Look values; [ns] = 0, [ns + 1] = -inf
        // the row's LSE folded in: t = S scale log2(e) + table - lse log2(e) in one FFMA
        for (int s = 0; s <= a.n_slots; ++s) trow[s * kRows] -= lse2;
      }
      for (int s = 0; s < a.n_slots + 2; ++s) drow[s * kRows] = 0.f;
      row_sync<kDqRowThreads>();
    }
    const uint8_t* sbase = p.slots_packed + int64_t(qt) * a.n_col_tiles * kSlotTileBytes + half * 4096 + row * 16;
    bool ok = true;
    uint4 cur[2], nxt[2];
    if (use_bias) {
      nxt[0] = __ldg(reinterpret_cast<const uint4*>(sbase));
      nxt[1] = __ldg(reinterpret_cast<const uint4*>(sbase + 2048));
    }
    for (int j = 0; j < a.n_col_tiles; ++j) {
      const int st = j & 1;
      if (use_bias) {  // this tile's slot bytes (loaded one tile ahead); the next tile's in flight
        cur[0] = nxt[0];
        cur[1] = nxt[1];
        if (j + 1 < a.n_col_tiles) {
          const uint8_t* src = sbase + int64_t(j + 1) * kSlotTileBytes;
          nxt[0] = __ldg(reinterpret_cast<const uint4*>(src));
          nxt[1] = __ldg(reinterpret_cast<const uint4*>(src + 2048));
        }
      }
      if (!mbar_wait(&bars->s_full[st], (j >> 1) & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[32], dr[32];
      const uint32_t xcol = lane_base + st * 128 + 32 * half;
      load_scores<32>(xcol, xcol + 64, sr, dr);
      const int32_t k0 = j * kCols + 32 * half;
      // Slot sums take only pairs with a Look slot (byte < ns); "no bias" and
      // "past the end" pairs are the large majority away from the query's
      // neighbourhood, and their sums are discarded.  A warp whose 32 rows have
      // no slotted pair in this tile skips the read-add-writes altogether.
      bool slotted = false;
      if (use_bias) {
        const uint32_t lim = 0x01010101u * static_cast<uint32_t>(a.n_slots);
        const uint32_t m = __vcmpltu4(cur[0].x, lim) | __vcmpltu4(cur[0].y, lim) | __vcmpltu4(cur[0].z, lim) |
                           __vcmpltu4(cur[0].w, lim) | __vcmpltu4(cur[1].x, lim) | __vcmpltu4(cur[1].y, lim) |
                           __vcmpltu4(cur[1].z, lim) | __vcmpltu4(cur[1].w, lim);
        slotted = __any_sync(0xffffffffu, m != 0u);
      }
      uint32_t dw[16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float g[8];
        if (use_bias) {
          uint32_t sl[8];
          float tb[8];
#pragma unroll
          for (int e2 = 0; e2 < 8; ++e2) {
            const int e = 8 * c + e2;
            sl[e2] = __byte_perm((&cur[e >> 4].x)[(e & 15) >> 2], 0u, 0x4440u | (e & 3));
            tb[e2] = trow[sl[e2] * kRows];
          }
#pragma unroll
          for (int e2 = 0; e2 < 8; ++e2) {
            const int e = 8 * c + e2;
            const float pr = fast_exp2(fmaf(__uint_as_float(sr[e]), scale_log2, tb[e2]));
            g[e2] = pr * (__uint_as_float(dr[e]) - delta);
          }
          // each cell of this warpgroup's array has one writer (this thread): a plain
          // read-add-write (measured faster than red.shared.add.f32 here)
          if (slotted) {
            // in pairs: both cells are read before either is written (half the
            // dependent read-add-write chain); a pair on one slot adds both values
            // through the first element (the second stores the cell unchanged first)
            const uint32_t ns = static_cast<uint32_t>(a.n_slots);
#pragma unroll
            for (int e2 = 0; e2 < 8; e2 += 2) {
              const uint32_t s0 = sl[e2], s1 = sl[e2 + 1];
              const bool r0 = s0 < ns, r1 = s1 < ns, same = s0 == s1;
              const float v0 = r0 ? drow[s0 * kRows] : 0.f;
              const float v1 = r1 ? drow[s1 * kRows] : 0.f;
              if (r1) drow[s1 * kRows] = v1 + (same ? 0.f : g[e2 + 1]);
              if (r0) drow[s0 * kRows] = v0 + g[e2] + (same ? g[e2 + 1] : 0.f);
            }
          }
        } else {
#pragma unroll
          for (int e2 = 0; e2 < 8; ++e2) {
            const int e = 8 * c + e2;
            const float t = k0 + e < N ? __uint_as_float(sr[e]) * scale_log2 : -INFINITY;
            g[e2] = fast_exp2(t - lse2) * (__uint_as_float(dr[e]) - delta);
          }
        }
#pragma unroll
        for (int e2 = 0; e2 < 8; e2 += 2) dw[4 * c + e2 / 2] = pk2<BF16>(g[e2], g[e2 + 1]);
      }
      tmem_st16(xcol, dw);  // dS, 16-bit, over this thread's already-read score columns
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ready[st]);
    }
    if (ok && !mbar_wait(&bars->acc_full, 0, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns)) ok = false;
    tc_fence_after();
    // dQ through shared memory: the Q / dO tiles are free once the last MMA is done
    float* dq_blk = reinterpret_cast<float*>(q_s);
    if (ok) {
      uint32_t q0[16], q1[16];
      tmem_ld16(lane_base + kColAcc0 + 32 * half, q0);
      tmem_ld16(lane_base + kColAcc0 + 32 * half + 16, q1);
      tmem_wait_ld();
      reg_fence16(q0);
      reg_fence16(q1);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        *blk_chunk(dq_blk, row, 8 * half + c) =
            make_float4(__uint_as_float(q0[4 * c]) * p.scale, __uint_as_float(q0[4 * c + 1]) * p.scale,
                        __uint_as_float(q0[4 * c + 2]) * p.scale, __uint_as_float(q0[4 * c + 3]) * p.scale);
        *blk_chunk(dq_blk, row, 8 * half + 4 + c) =
            make_float4(__uint_as_float(q1[4 * c]) * p.scale, __uint_as_float(q1[4 * c + 1]) * p.scale,
                        __uint_as_float(q1[4 * c + 2]) * p.scale, __uint_as_float(q1[4 * c + 3]) * p.scale);
      }
    }
    row_sync<kDqRowThreads>();  // dQ staged; both warpgroups' slot sums are in
    const int tile_rows = N - qt * kRows < kRows ? N - qt * kRows : kRows;
    if (ok && a.grad_q != nullptr)
      blk_copy_out(dq_blk, a.grad_q + (int64_t(bh) * N + qt * kRows) * D64, tile_rows, threadIdx.x, kDqRowThreads);
    if (use_bias) {
      // slot gradient rows [row][slot] (odd row stride: conflict-free per-row writes) in
      // the Look table's place, then copied out slot-contiguously
      const int ns = a.n_slots, pst = ns | 1;
      float* pblk = table_s;
      if (ok && half == 0) {
        const float* other = drow + (ns + 2) * kRows;
        for (int s = 0; s < ns; ++s) pblk[row * pst + s] = drow[s * kRows] + other[s * kRows];
      }
      row_sync<kDqRowThreads>();
      if (ok && a.grad_pose != nullptr) {
        for (int idx = threadIdx.x; idx < tile_rows * ns; idx += kDqRowThreads) {
          const int r = idx / ns, sl = idx - r * ns;
          const int32_t tok = qt * kRows + r;
          if (tok >= 1) a.grad_pose[((int64_t(b) * (N - 1) + (tok - 1)) * H + h) * ns + sl] = pblk[r * pst + sl];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kDqMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================================ dK, dV
// Stage block of one 64-query tile: table[64][table_w] (the queries' Look
// values as stored; table_w = round_up(ns + 2, 4); column ns = 0 ("no bias")
// and column ns + 1 = -inf (query past the end), both written once per CTA),
// then lse [64], then delta [64].  Thread t copies query row t / 8 (its
// 16-byte slot groups t % 8 + 8m, or its slots t % 8 + 8m one by one when the
// rows are not 16-byte aligned) and, for t < 128, one lse / delta value, with
// cp.async straight into shared memory two tiles ahead, and hands the copies'
// completion to the block's stage_full barrier (cp.async.mbarrier.arrive).
// The log2(e) scaling and the query's lse are applied where the values are
// used (t = S scale log2 e + (v - lse) log2 e), so no thread rewrites a block
// and the row threads never meet at a CTA-wide barrier: a block is reused
// once every row warp has arrived on its stage_free barrier.  Rows and
// queries outside 1..N-1 / 0..N-1 are zero-filled (the slot table sends those
// pairs to the constant columns).
constexpr int kKvThreads = kKvRowThreads + 32;
constexpr int kKvMmaWarp = kKvRowThreads / 32;
constexpr int kStageLanes = kKvRowThreads / kCols;  // threads per query row: 8
constexpr int kMaxStageVec = (kMaxLookSlots / 4 + kStageLanes - 1) / kStageLanes;
constexpr int kMaxStageScalar = (kMaxLookSlots + kStageLanes - 1) / kStageLanes;

__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool pred) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(pred ? 4 : 0)
               : "memory");
}
// Arrive on `bar` once this thread's earlier cp.async copies have landed (the
// barrier's count includes this arrival: .noinc).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Issues this thread's copies of tile (q0..q0+63)'s stage block.
template <class A>
__device__ __forceinline__ void stage_issue(float* blk, const A& a, int tid, int32_t q0, int64_t b, int64_t h) {
  const SlaParams& p = a.p;
  const int32_t N = static_cast<int32_t>(p.seq);
  const int ns = a.n_slots, tw = a.table_w;
  const int q = tid / kStageLanes, c = tid % kStageLanes;
  const int32_t tok = q0 + q;
  const bool valid = tok >= 1 && tok < N;
  if (ns > 0) {
    const float* pose = static_cast<const float*>(p.pose);
    const float* src = pose + b * p.pose_stride[0] + int64_t(valid ? tok - 1 : 0) * p.pose_stride[1] +
                       h * p.pose_stride[2];
    float* row = blk + q * tw;
    if (a.pose_vec4) {
#pragma unroll
      for (int m = 0; m < kMaxStageVec; ++m) {
        const int g = c + kStageLanes * m;
        if (g < ns / 4) cp_async16(row + 4 * g, src + 4 * g, valid);
      }
    } else {
#pragma unroll 4
      for (int m = 0; m < kMaxStageScalar; ++m) {
        const int sl = c + kStageLanes * m;
        if (sl < ns) cp_async4(row + sl, src + sl, valid);
      }
    }
  }
  const int64_t bh_off = (b * p.heads + h) * N;
  if (tid < 2 * kCols) {
    const int32_t tq = q0 + (tid & (kCols - 1));
    const float* base = tid < kCols ? p.lse : a.delta;
    cp_async4(blk + kCols * tw + tid, base + bh_off + (tq < N ? tq : 0), tq < N);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(kKvThreads, 1)
sla_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                    const FusedArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* k_s = smem;
  uint8_t* v_s = smem + kTileRows;
  uint8_t* q_s = smem + 2 * kTileRows;
  uint8_t* do_s = q_s + kStages * kTileCols;
  float* stage_s = reinterpret_cast<float*>(smem + a.off_table);  // kStageBufs stage blocks
  FusedBars* bars = reinterpret_cast<FusedBars*>(smem + a.off_bars);
  const SlaParams& p = a.p;
  volatile int32_t* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t H = static_cast<uint32_t>(p.heads);
  const int32_t N = static_cast<int32_t>(p.seq);
  const int32_t kt = static_cast<int32_t>(blockIdx.x % a.n_row_tiles);
  const uint32_t bh = blockIdx.x / a.n_row_tiles;
  const int32_t h = static_cast<int32_t>(bh % H), b = static_cast<int32_t>(bh / H);
  const bool use_bias = a.n_slots > 0;
  const int tw = a.table_w;
  const int stage_n = kCols * tw + 2 * kCols;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStageBufs; ++s) {
      mbar_init(&bars->stage_full[s], kKvRowThreads);
      mbar_init(&bars->stage_free[s], kKvRowThreads / 32);
    }
    init_bars(bars, kKvRowThreads / 32);
  }
  if (warp == kKvMmaWarp) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kKvMmaWarp) {
    if (lane == 0)
      mma_role<BF16, true, 16>(&tm_k, &tm_v, &tm_q, &tm_do, a, bars, k_s, v_s, q_s, do_s, tmem, kt, h, b);
  } else {
    const int tid = threadIdx.x;
    const int row = tid & (kRows - 1);
    const int wg = tid >> 7;                  // query columns 16 wg .. 16 wg + 15 of each tile
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float scale_log2 = p.scale * kLog2eF;
    const int n_t = a.n_col_tiles;
    // the constant columns of every block, then tiles 0 and 1 in flight
    if (use_bias && tid < kStageBufs * kCols) {
      float* crow = stage_s + (tid / kCols) * stage_n + (tid % kCols) * tw + a.n_slots;
      crow[0] = 0.f;
      crow[1] = -INFINITY;
    }
    row_sync<kKvRowThreads>();
    stage_issue(stage_s, a, tid, 0, b, h);
    cp_async_arrive(&bars->stage_full[0]);
    if (n_t > 1) {
      stage_issue(stage_s + stage_n, a, tid, kCols, b, h);
      cp_async_arrive(&bars->stage_full[1]);
    }
    const uint8_t* sbase = a.slots_t + int64_t(kt) * n_t * kSlotTileBytes + wg * 2048 + row * 16;
    uint4 cur, nxt;
    if (use_bias) nxt = __ldg(reinterpret_cast<const uint4*>(sbase));
    bool ok = true;
    for (int t = 0; t < n_t; ++t) {
      const int st = t & 1, sb = t % kStageBufs;
      const float* blk = stage_s + sb * stage_n;
      // tile t + 2's stage block into the block tile t - 1 used, once every row warp has read it
      if (t + 2 < n_t) {
        const int nb = (t + 2) % kStageBufs;
        if (t >= 1 && !mbar_wait(&bars->stage_free[nb], ((t - 1) / kStageBufs) & 1, abort_flag, p.status,
                                 kDevTimeoutSoftmax, a.wait_ns)) {
          ok = false;
          break;
        }
        stage_issue(stage_s + nb * stage_n, a, tid, (t + 2) * kCols, b, h);
        cp_async_arrive(&bars->stage_full[nb]);
      }
      if (use_bias) {  // this tile's slot bytes (loaded one tile ahead); the next tile's in flight
        cur = nxt;
        if (t + 1 < n_t) nxt = __ldg(reinterpret_cast<const uint4*>(sbase + int64_t(t + 1) * kSlotTileBytes));
      }
      if (!mbar_wait(&bars->s_full[st], (t >> 1) & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns) ||
          !mbar_wait(&bars->stage_full[sb], (t / kStageBufs) & 1, abort_flag, p.status, kDevTimeoutSoftmax,
                     a.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[16], dr[16];
      const uint32_t xcol = lane_base + st * 128 + 16 * wg;
      load_scores<16>(xcol, xcol + 64, sr, dr);
      const float4* lse4 = reinterpret_cast<const float4*>(blk + kCols * tw + 16 * wg);
      const float4* dlt4 = lse4 + kCols / 4;
      const float* tab = blk + 16 * wg * tw;
      const int32_t qbase = t * kCols + 16 * wg;
      uint32_t pw[8], dw[8];
#pragma unroll
      for (int e4 = 0; e4 < 16; e4 += 4) {
        const float4 d4 = dlt4[e4 / 4], l4 = lse4[e4 / 4];
        const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
        float tl[4];
        if (use_bias) {
          const uint32_t word = (&cur.x)[e4 >> 2];
#pragma unroll
          for (int u = 0; u < 4; ++u) tl[u] = tab[(e4 + u) * tw + __byte_perm(word, 0u, 0x4440u | u)];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            tl[u] = fmaf(__uint_as_float(sr[e4 + u]), scale_log2, (tl[u] - lv[u]) * kLog2eF);
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            tl[u] = qbase + e4 + u < N ? fmaf(__uint_as_float(sr[e4 + u]), scale_log2, -lv[u] * kLog2eF) : -INFINITY;
        }
        float pr[4], gg[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          pr[u] = fast_exp2(tl[u]);
          gg[u] = pr[u] * (__uint_as_float(dr[e4 + u]) - dv[u]);
        }
        pw[e4 / 2] = pk2<BF16>(pr[0], pr[1]);
        pw[e4 / 2 + 1] = pk2<BF16>(pr[2], pr[3]);
        dw[e4 / 2] = pk2<BF16>(gg[0], gg[1]);
        dw[e4 / 2 + 1] = pk2<BF16>(gg[2], gg[3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->stage_free[sb]);  // this warp is through with the block
      tmem_st8(xcol, pw);        // P^T over the read score columns
      tmem_st8(xcol + 64, dw);   // dS^T over the read dP columns
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ready[st]);
    }
    cp_async_wait_all();  // no copy of this thread is still in flight past this point
    if (ok && !mbar_wait(&bars->acc_full, 0, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns)) ok = false;
    tc_fence_after();
    // dK and dV through shared memory: the K / V tiles and the ring are free once the last MMA is done
    float* dk_blk = reinterpret_cast<float*>(smem);
    float* dv_blk = dk_blk + kRows * D64;
    if (ok) {
      uint32_t kr[16], vr[16];
      tmem_ld16(lane_base + kColAcc0 + 16 * wg, kr);
      tmem_ld16(lane_base + kColAcc1 + 16 * wg, vr);
      tmem_wait_ld();
      reg_fence16(kr);
      reg_fence16(vr);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        *blk_chunk(dk_blk, row, 4 * wg + c) =
            make_float4(__uint_as_float(kr[4 * c]) * p.scale, __uint_as_float(kr[4 * c + 1]) * p.scale,
                        __uint_as_float(kr[4 * c + 2]) * p.scale, __uint_as_float(kr[4 * c + 3]) * p.scale);
        *blk_chunk(dv_blk, row, 4 * wg + c) = make_float4(__uint_as_float(vr[4 * c]), __uint_as_float(vr[4 * c + 1]),
                                                          __uint_as_float(vr[4 * c + 2]), __uint_as_float(vr[4 * c + 3]));
      }
    }
    row_sync<kKvRowThreads>();
    const int tile_rows = N - kt * kRows < kRows ? N - kt * kRows : kRows;
    const int64_t off = (int64_t(bh) * N + kt * kRows) * D64;
    if (ok && a.grad_k != nullptr) blk_copy_out(dk_blk, a.grad_k + off, tile_rows, tid, kKvRowThreads);
    if (ok && a.grad_v != nullptr) blk_copy_out(dv_blk, a.grad_v + off, tile_rows, tid, kKvRowThreads);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kKvMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

uint32_t round_up(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }

}  // namespace

int32_t sla_backward_fused_supported(const SlaBwdParams& bp, const uint8_t* slots_t) {
  const SlaParams& p = bp.f;
  if (!tc_common_ok(p)) return 0;
  if (p.dense != nullptr || bp.grad_fields != nullptr || bp.grad_dense != nullptr) return 0;
  if (p.bias_mode != 0 && p.bias_mode != 2) return 0;
  if (p.bias_mode == 2 && (p.poses < 1 || p.poses > kMaxLookSlots || !p.slots_packed || !slots_t)) return 0;
  // the dK / dV kernel copies pose rows with cp.async: fp32, unit stride along slots
  if (p.bias_mode == 2 && (p.pose_dtype != 0 || p.pose_stride[3] != 1 || reinterpret_cast<uintptr_t>(p.pose) % 4))
    return 0;
  if (!p.lse || !bp.grad_out || !bp.delta) return 0;
  if (!tma_stride_ok(bp.grad_out, bp.grad_out_stride)) return 0;
  for (float* g : {bp.grad_q, bp.grad_k, bp.grad_v})
    if (g != nullptr && reinterpret_cast<uintptr_t>(g) % 16) return 0;
  return 1;
}

int32_t launch_sla_backward_fused(const SlaBwdParams& bp, const uint8_t* slots_t, cudaStream_t stream) {
  if (!sla_backward_fused_supported(bp, slots_t)) return 8;
  const SlaParams& p = bp.f;
  FusedArgs a;
  a.p = p;
  a.dout = bp.grad_out;
  for (int d = 0; d < 4; ++d) a.dout_stride[d] = bp.grad_out_stride[d];
  a.grad_q = bp.grad_q;
  a.grad_k = bp.grad_k;
  a.grad_v = bp.grad_v;
  a.grad_pose = bp.grad_pose;
  a.delta = bp.delta;
  a.slots_t = slots_t;
  a.n_slots = p.bias_mode == 2 ? static_cast<int32_t>(p.poses) : 0;
  a.table_w = a.n_slots > 0 ? static_cast<int32_t>(round_up(static_cast<uint32_t>(a.n_slots + 2), 4)) : 0;
  a.pose_vec4 = (p.bias_mode == 2 && p.pose_dtype == 0 && p.pose_stride[3] == 1 && a.n_slots % 4 == 0 &&
                 reinterpret_cast<uintptr_t>(p.pose) % 16 == 0 && p.pose_stride[0] % 4 == 0 &&
                 p.pose_stride[1] % 4 == 0 && p.pose_stride[2] % 4 == 0)
                    ? 1 : 0;
  a.wait_ns = tc_wait_budget_ns();
  const int32_t n128 = static_cast<int32_t>((p.seq + kRows - 1) / kRows);
  const int32_t n64 = static_cast<int32_t>((p.seq + kCols - 1) / kCols);
  const int64_t grid = p.batch * p.heads * n128;
  if (grid > INT32_MAX) return 8;
  a.n_row_tiles = n128;
  a.n_col_tiles = n64;
  CUtensorMap m_q128, m_do128, m_k64, m_v64, m_k128, m_v128, m_q64, m_do64;
  MapOrder o[8];
  if (!make_map(&m_q128, &o[0], p.q, p.q_stride, p, kRows) ||
      !make_map(&m_do128, &o[1], bp.grad_out, bp.grad_out_stride, p, kRows) ||
      !make_map(&m_k64, &o[2], p.k, p.k_stride, p, kCols) || !make_map(&m_v64, &o[3], p.v, p.v_stride, p, kCols) ||
      !make_map(&m_k128, &o[4], p.k, p.k_stride, p, kRows) || !make_map(&m_v128, &o[5], p.v, p.v_stride, p, kRows) ||
      !make_map(&m_q64, &o[6], p.q, p.q_stride, p, kCols) ||
      !make_map(&m_do64, &o[7], bp.grad_out, bp.grad_out_stride, p, kCols))
    return 4;

  // dQ, delta and the slot gradient
  {
    FusedArgs q = a;
    q.o_fixed0 = o[0];
    q.o_fixed1 = o[1];
    q.o_ring0 = o[2];
    q.o_ring1 = o[3];
    const uint32_t table_bytes = q.n_slots > 0 ? static_cast<uint32_t>((q.n_slots + 2) * kRows * 4) : 0u;
    uint32_t off = 2 * kTileRows + 2 * kStages * kTileCols;
    q.off_table = off;
    off += table_bytes;
    q.off_dacc = off;
    off += 2 * table_bytes;
    q.off_bars = round_up(off, 64);
    size_t smem = q.off_bars + sizeof(FusedBars) + 1024;
    if (smem < kMinSmem) smem = kMinSmem;
    auto kernel = p.dtype == 2 ? sla_bwd_dq_kernel<true> : sla_bwd_dq_kernel<false>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return 6;
    kernel<<<static_cast<unsigned>(grid), kDqThreads, smem, stream>>>(m_q128, m_do128, m_k64, m_v64, q);
    if (cudaGetLastError() != cudaSuccess) return 6;
  }
  if (bp.grad_k == nullptr && bp.grad_v == nullptr) return 0;
  // dK, dV
  {
    FusedArgs kv = a;
    kv.o_fixed0 = o[4];
    kv.o_fixed1 = o[5];
    kv.o_ring0 = o[6];
    kv.o_ring1 = o[7];
    const uint32_t stage_bytes = static_cast<uint32_t>((kCols * kv.table_w + 2 * kCols) * 4);
    uint32_t off = 2 * kTileRows + 2 * kStages * kTileCols;
    kv.off_table = off;
    kv.off_dacc = off;
    off += kStageBufs * stage_bytes;
    kv.off_bars = round_up(off, 64);
    size_t smem = kv.off_bars + sizeof(FusedBars) + 1024;
    if (smem < kMinSmem) smem = kMinSmem;
    auto kernel = p.dtype == 2 ? sla_bwd_dkdv_kernel<true> : sla_bwd_dkdv_kernel<false>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return 6;
    kernel<<<static_cast<unsigned>(grid), kKvThreads, smem, stream>>>(m_k128, m_v128, m_q64, m_do64, kv);
    if (cudaGetLastError() != cudaSuccess) return 6;
  }
  return 0;
}

}  // namespace intp
