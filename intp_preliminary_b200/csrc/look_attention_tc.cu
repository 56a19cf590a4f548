// look_attention_tc.cu - tcgen05 / TMA structured Look attention forward (sm_100a).
//
// Semantics: layers/triton_structured_look_attention.py:25-54 (oracle) and
// :57-169 (the reference's Triton forward), for bf16 / f16 inputs, head_dim 64,
// with the Look bias in SLOTS form (bias[b,h,i,j] = pose[b,i-1,h,slot(i,j)],
// the one-hot-fields case of the reference API), in SLOT_FIELDS form
// (bias = sum_p pose[b,i-1,h,p] * slot_fields[h,p,slot(i,j)]: the reference
// model's fields, stored per slot) or without bias.  Either Look form becomes
// a per-query table of slot values in shared memory at the start of a work
// item; the score tiles then gather from it by the packed pair table.
//
// CTA organisation (192 threads, two CTAs per SM):
//   warps 0-3  softmax warpgroup: thread t owns query row t of the 128-row tile.
//              Reads S from TMEM, adds the Look bias from shared memory, runs the
//              online softmax in the log2 domain and writes P (16-bit) back into
//              the same TMEM columns S came from.  O is rescaled in TMEM only
//              when the running max grows by more than 2^8.  At the end of an
//              item it normalises O and stores it (plus the LSE).
//   warp 4     TMA producer: Q tile (128 x 64) per work item, then K tiles of
//              64 keys with their 8 KB packed slot tiles (3-stage ring, freed
//              once S(j) is computed and its slots are read) and V tiles
//              (2-stage ring, freed once PV(j) completes).
//   warp 5     MMA issuer: S = Q K^T (tcgen05.mma kind::f16, both operands in
//              shared memory, accumulator in TMEM) and O += P [V | 1] with P read
//              from TMEM.  The extra B block is a constant column of ones, so O
//              column 64 accumulates the softmax row sum on the tensor core.
// TMEM columns: [0,64) S / P buffer 0, [64,128) S / P buffer 1, [128,208) O
// (64 output columns + the row-sum column + 15 unused).  An S buffer is reused
// for tile j+2 only after PV(j), which reads P(j) from it, has completed.
//
// The CTA is persistent over work items (batch, head, 128-row query tile).
// Every mbarrier wait is bounded (sm100_ptx.cuh); on expiry the CTA unwinds,
// drains its own in-flight copies and MMAs, frees TMEM and reports through the
// status word instead of hanging.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "sla_internal.h"
#include "sm100_ptx.cuh"
#include "tma_host.h"
#include "sla_tc_common.cuh"
#include "sla_look_table.cuh"

namespace intp {
namespace {

constexpr int BM = 128;            // query rows per tile
constexpr int BN = 64;             // keys per tile
constexpr int HD = 64;             // head_dim
constexpr int ON = HD + 16;        // PV MMA N: 64 outputs + the ones block (row sum in column 64)
constexpr int kThreads = 192;
constexpr int kVStages = 2;   // V tile ring (released after PV(j))
constexpr uint32_t kQBytes = BM * HD * 2;      // 16 KB
constexpr uint32_t kKVBytes = BN * HD * 2;     // 8 KB each of K and V (and the ones tile)
constexpr uint32_t kSlotBytes = kSlotTileBytes;  // 8 KB
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS0 = 0, kColS1 = 64, kColO = 128;
constexpr float kLog2e = kLog2eF;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P values stay <= 2^8
constexpr int kFmaExpPairs = 8;            // of a tile's 32 key pairs: exponentials on the FMA pipe
constexpr int kMaxSlots = kMaxLookSlots;
constexpr int kMaxPoses = kMaxLookPoses;
template <int KS>
struct alignas(8) Barriers {
  uint64_t q_full, q_empty;
  uint64_t k_full[KS], k_empty[KS];
  uint64_t v_full[kVStages], v_empty[kVStages];
  // s_full[b]: S of a tile is in buffer b.  p_full[b]: its P is stored there.
  // pv_done[b]: the PV that read that P finished (buffer b is free again).
  // One barrier per buffer keeps every waiter at most one phase behind.
  uint64_t s_full[2], p_full[2], pv_done[2];
  uint64_t sf_ready;  // SLOT_FIELDS: an item's slot values are staged (4 softmax warps)
  uint64_t sf_free;   // SLOT_FIELDS: the 4 softmax warps built that item's table
  uint64_t drain;
  uint32_t tmem_base;
  int32_t abort;
};

// KS = stages of the K / slot-tile ring: 3 normally, 2 when the per-query
// Look table is large (keeps two CTAs per SM).
template <int KS>
struct SmemLayout {
  // offsets relative to a 1024-byte aligned base
  static constexpr uint32_t q = 0;
  static constexpr uint32_t k = q + kQBytes;
  static constexpr uint32_t v = k + KS * kKVBytes;
  static constexpr uint32_t ones = v + kVStages * kKVBytes;  // constant [keys][64] tile, column 0 = 1
  static constexpr uint32_t slots = ones + kKVBytes;
  static constexpr uint32_t table = slots + KS * kSlotBytes;
};

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Row maximum of 64 values (32 pairs) as a shallow tree of three-input maxima.
__device__ __forceinline__ float row_max64(const float2 (&t)[32]) {
  float m8[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float2* v = t + 4 * k;
    m8[k] = fmaxf(fmax3(fmax3(v[0].x, v[0].y, v[1].x), fmax3(v[1].y, v[2].x, v[2].y), v[3].x), v[3].y);
  }
  return fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack_out(uint32_t lo, uint32_t hi, float inv) {
  return pack2<BF16>(__uint_as_float(lo) * inv, __uint_as_float(hi) * inv);
}

// P = 2^(t * cs - m) for the 64 keys of a row, packed to 16-bit pairs in key
// order.  Eight of the 32 pairs are exponentiated on the FMA pipe (exp2_fma),
// the rest on the MUFU: the softmax is bound by its exponentials, and that
// share measured fastest (cfg4-shaped layer: 279.6 -> 272.6 us).
template <bool BF16>
__device__ __forceinline__ void exp_pack(const float2 (&t)[BN / 2], float cs, float m, uint32_t (&w)[BN / 2]) {
  const float2 c2 = make_float2(cs, cs), nm2 = make_float2(-m, -m);
#pragma unroll
  for (int c = 0; c < BN / 2; ++c) {
    const float2 x = fma2(t[c], c2, nm2);
    const float2 p = (c & 1) && (c >> 1) < kFmaExpPairs ? exp2_fma(x) : make_float2(fast_exp2(x.x), fast_exp2(x.y));
    w[c] = pack2<BF16>(p.x, p.y);
  }
}

struct TcArgs {
  SlaParams p;
  MapOrder oq, ok, ov;
  int64_t n_qt, n_kt, n_items;
  int32_t n_slots;        // 0 when there is no Look bias
  uint32_t table_bytes;   // bytes of the per-query Look table in smem
  int32_t pose_vec4;      // pose rows are 16-byte aligned fp32 with unit stride along slots
                          // (SLOTS) or poses (SLOT_FIELDS, poses % 4 == 0)
  int32_t slot_fields;    // 1: SLOT_FIELDS mode (table = pose . slot_fields)
  int32_t n_poses;        // SLOT_FIELDS: poses per head
  int32_t sf_vec4;        // SLOT_FIELDS: slot_fields rows are 16-byte aligned fp32, unit slot stride;
                          // the head's rows are then staged in smem after the table
  uint32_t sf_offset;     // SLOT_FIELDS with sf_vec4: floats from the table start to the staged rows
  uint64_t wait_ns;       // budget of the pipeline waits (drains keep the default)
};

// S row (64 fp32 scores of this thread's TMEM lane) into t[c] = keys 2c, 2c+1.
__device__ __forceinline__ void load_s_row(uint32_t s_addr, float2 (&t)[BN / 2]) {
  uint32_t r0[16], r1[16], r2[16], r3[16];
  tmem_ld16(s_addr, r0);
  tmem_ld16(s_addr + 16, r1);
  tmem_ld16(s_addr + 32, r2);
  tmem_ld16(s_addr + 48, r3);
  tmem_wait_ld();
  reg_fence16(r0);
  reg_fence16(r1);
  reg_fence16(r2);
  reg_fence16(r3);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    t[e] = make_float2(__uint_as_float(r0[2 * e]), __uint_as_float(r0[2 * e + 1]));
    t[8 + e] = make_float2(__uint_as_float(r1[2 * e]), __uint_as_float(r1[2 * e + 1]));
    t[16 + e] = make_float2(__uint_as_float(r2[2 * e]), __uint_as_float(r2[2 * e + 1]));
    t[24 + e] = make_float2(__uint_as_float(r3[2 * e]), __uint_as_float(r3[2 * e + 1]));
  }
}

// t = scale*log2(e)*s + bias (log2 domain): slot bytes from the packed tile row,
// per-query values from the [slot][row] table.
__device__ __forceinline__ void add_look_bias(float2 (&t)[BN / 2], const uint8_t* srow, const float* trow,
                                              float scale_log2) {
#pragma unroll
  for (int c = 0; c < BN / 16; ++c) {
    const uint4 w = *reinterpret_cast<const uint4*>(srow + c * 2048);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      const uint32_t s0 = __byte_perm(ww[e >> 2], 0u, 0x4440u | (e & 3));
      const uint32_t s1 = __byte_perm(ww[e >> 2], 0u, 0x4440u | ((e + 1) & 3));
      float2& tv = t[c * 8 + e / 2];
      tv.x = fmaf(tv.x, scale_log2, trow[s0 * BM]);
      tv.y = fmaf(tv.y, scale_log2, trow[s1 * BM]);
    }
  }
}

// The constant "ones" tile: 64 keys x 64 columns (16-bit) in the 128B-swizzled
// layout TMA gives V, logical column 0 = 1, every other column 0.  Written by
// 128 threads (thread index `tid`).
template <bool BF16>
__device__ __forceinline__ void fill_ones_tile(uint8_t* ones_s, int tid) {
  const uint16_t one = BF16 ? uint16_t(0x3F80) : uint16_t(0x3C00);
  for (int w = tid; w < static_cast<int>(kKVBytes / 16); w += 128) {
    const int r = w >> 3, chunk = w & 7;  // 16-byte chunk `chunk` of key row r
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (chunk == (r & 7)) v.x = one;      // logical chunk 0 lands at physical chunk r % 8
    reinterpret_cast<uint4*>(ones_s)[w] = v;
  }
  fence_proxy_async_shared();  // generic-proxy writes -> visible to the tensor core
}

template <int KS, bool BF16>
__global__ void __launch_bounds__(kThreads, 2)
sla_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  using Layout = SmemLayout<KS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment (128B-swizzle tiles) by an offset from the __shared__
  // array itself, so every derived pointer stays in the shared address space
  // (32-bit LDS/STS instead of generic 64-bit loads).
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Barriers<KS>* bars = reinterpret_cast<Barriers<KS>*>(smem + Layout::table + a.table_bytes);
  uint8_t* q_s = smem + Layout::q;
  uint8_t* k_s = smem + Layout::k;
  uint8_t* v_s = smem + Layout::v;
  uint8_t* ones_s = smem + Layout::ones;
  uint8_t* slot_s = smem + Layout::slots;
  float* table_s = reinterpret_cast<float*>(smem + Layout::table);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const SlaParams& p = a.p;
  volatile int32_t* abort_flag = &bars->abort;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1 + 4);  // S-MMA commit + 4 softmax warps (slot reads)
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);  // PV-MMA commit
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_full[s], 4);
      mbar_init(&bars->pv_done[s], 1);
    }
    mbar_init(&bars->sf_ready, 4);
    mbar_init(&bars->sf_free, 4);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    mbar_fence_init();
  }
  if (warp < 4) fill_ones_tile<BF16>(ones_s, threadIdx.x);
  if (warp == 5) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  // Work-item indices fit 32 bits (checked on the host): 32-bit divisions.
  const int64_t N = p.seq;
  const uint32_t H = static_cast<uint32_t>(p.heads);
  const int64_t n_kt = a.n_kt;
  const uint32_t n_qt = static_cast<uint32_t>(a.n_qt), n_items = static_cast<uint32_t>(a.n_items);
  const bool use_bias = a.n_slots > 0;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    // K tiles (with their slot tiles) run up to KS ahead; V tiles lag one
    // key tile behind K so a V stage still in use never blocks the next K load.
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      uint32_t k_iter = 0, v_iter = 0, item_iter = 0;
      bool ok = true;
      auto load_v = [&](int64_t jv, int32_t h, int32_t b) -> bool {
        const uint32_t vs = v_iter % kVStages, n = v_iter / kVStages;
        if (n > 0 && !mbar_wait(&bars->v_empty[vs], (n - 1) & 1, abort_flag, p.status, kDevTimeoutProducer, a.wait_ns))
          return false;
        mbar_arrive_expect_tx(&bars->v_full[vs], kKVBytes);
        const int32_t r = static_cast<int32_t>(jv * BN);
        tma_load_4d(v_s + vs * kKVBytes, &tm_v, &bars->v_full[vs], 0, map_coord(a.ov, 1, r, h, b),
                    map_coord(a.ov, 2, r, h, b), map_coord(a.ov, 3, r, h, b));
        ++v_iter;
        return true;
      };
      for (uint32_t item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_iter) {
        const uint32_t qt = item % n_qt;
        const uint32_t bh = item / n_qt;
        const int32_t h = static_cast<int32_t>(bh % H), b = static_cast<int32_t>(bh / H);
        if (item_iter > 0 && !mbar_wait(&bars->q_empty, (item_iter - 1) & 1, abort_flag, p.status,
                                        kDevTimeoutProducer, a.wait_ns)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars->q_full, kQBytes);
        {
          const int32_t r = static_cast<int32_t>(qt * BM);
          tma_load_4d(q_s, &tm_q, &bars->q_full, 0, map_coord(a.oq, 1, r, h, b), map_coord(a.oq, 2, r, h, b),
                      map_coord(a.oq, 3, r, h, b));
        }
        for (int64_t j = 0; j < n_kt; ++j) {
          const uint32_t ks = k_iter % KS, n = k_iter / KS;
          if (n > 0 && !mbar_wait(&bars->k_empty[ks], (n - 1) & 1, abort_flag, p.status, kDevTimeoutProducer, a.wait_ns)) {
            ok = false;
            break;
          }
          const bool bias_tile = use_bias && p.slot_tile_flags[qt * n_kt + j];
          mbar_arrive_expect_tx(&bars->k_full[ks], kKVBytes + (bias_tile ? kSlotBytes : 0));
          const int32_t r = static_cast<int32_t>(j * BN);
          tma_load_4d(k_s + ks * kKVBytes, &tm_k, &bars->k_full[ks], 0, map_coord(a.ok, 1, r, h, b),
                      map_coord(a.ok, 2, r, h, b), map_coord(a.ok, 3, r, h, b));
          if (bias_tile)
            bulk_load(slot_s + ks * kSlotBytes, p.slots_packed + (qt * n_kt + j) * kSlotBytes, kSlotBytes,
                      &bars->k_full[ks]);
          ++k_iter;
          if (j > 0 && !load_v(j - 1, h, b)) {
            ok = false;
            break;
          }
        }
        if (ok && !load_v(n_kt - 1, h, b)) ok = false;
      }
      // Drain: never leave a copy in flight into shared memory of an exiting CTA.
      // Stage s of a ring with `issued` loads received (issued - s + R - 1) / R of them.
      volatile int32_t no_abort = 0;
      if (item_iter > 0) mbar_wait(&bars->q_full, (item_iter - 1) & 1, &no_abort, p.status, kDevTimeoutDrain);
      for (uint32_t st = 0; st < KS; ++st) {
        const uint32_t cnt = k_iter > st ? (k_iter - st + KS - 1) / KS : 0;
        if (cnt > 0) mbar_wait(&bars->k_full[st], (cnt - 1) & 1, &no_abort, p.status, kDevTimeoutDrain);
      }
      for (uint32_t st = 0; st < kVStages; ++st) {
        const uint32_t cnt = v_iter > st ? (v_iter - st + kVStages - 1) / kVStages : 0;
        if (cnt > 0) mbar_wait(&bars->v_full[st], (cnt - 1) & 1, &no_abort, p.status, kDevTimeoutDrain);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qk = idesc_f16(BF16, false, BM, BN);
      const uint32_t idesc_pv = idesc_f16(BF16, true, BM, ON);
      // Descriptors are built once; a K step / stage advances only the 14-bit
      // start-address field (16-byte units) in the low word, which cannot carry.
      // V is MN-major with two 64-wide column blocks: the V tile and, LBO bytes
      // further, the constant ones tile.
      const uint32_t v_addr = smem_u32(v_s), ones_addr = smem_u32(ones_s);
      const uint64_t q_desc = smem_desc_sw128(smem_u32(q_s), 16, 1024);
      const uint64_t k_desc = smem_desc_sw128(smem_u32(k_s), 16, 1024);
      const uint64_t v_desc0 = smem_desc_sw128(v_addr, ones_addr - v_addr, 1024);
      const uint64_t v_desc1 = smem_desc_sw128(v_addr + kKVBytes, ones_addr - (v_addr + kKVBytes), 1024);
      uint32_t k_iter = 0, v_iter = 0, s_iter = 0, pv_iter = 0, item_iter = 0;
      bool ok = true, issued = false;
      // O += P [V | 1] for the tile whose P the softmax just published (global tile pv_iter).
      auto issue_pv = [&](bool first_tile) -> bool {
        const uint32_t pb = pv_iter & 1;
        if (!mbar_wait(&bars->p_full[pb], (pv_iter >> 1) & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) return false;
        const uint32_t vs = v_iter % kVStages;
        if (!mbar_wait(&bars->v_full[vs], (v_iter / kVStages) & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns))
          return false;
        tc_fence_after();
        const uint64_t vd = vs == 0 ? v_desc0 : v_desc1;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_ts(tmem + kColO, tmem + (pb ? kColS1 : kColS0) + kk * 8, vd + ((kk * 2048) >> 4), idesc_pv,
                 (!first_tile || kk > 0) ? 1u : 0u);
        mma_commit(&bars->pv_done[pb]);
        mma_commit(&bars->v_empty[vs]);
        ++pv_iter;
        ++v_iter;
        return true;
      };
      for (uint32_t item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_iter) {
        if (!mbar_wait(&bars->q_full, item_iter & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int64_t j = 0; j < n_kt && ok; ++j) {
          const uint32_t ks = k_iter % KS;
          if (!mbar_wait(&bars->k_full[ks], (k_iter / KS) & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) {
            ok = false;
            break;
          }
          // S buffer sb last held P of tile s_iter - 2: its PV must be done.
          const uint32_t sb = s_iter & 1;
          if (s_iter >= 2 &&
              !mbar_wait(&bars->pv_done[sb], ((s_iter - 2) >> 1) & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t s_col = tmem + (sb ? kColS1 : kColS0);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint64_t ad = q_desc + ((kk * 32) >> 4);
            const uint64_t bd = k_desc + ((ks * kKVBytes + kk * 32) >> 4);
            mma_ss(s_col, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          mma_commit(&bars->s_full[sb]);
          mma_commit(&bars->k_empty[ks]);
          issued = true;
          ++s_iter;
          ++k_iter;
          if (j > 0 && !issue_pv(j == 1)) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
        mma_commit(&bars->q_empty);
        if (!issue_pv(n_kt == 1)) {
          ok = false;
          break;
        }
      }
      // Drain: all issued MMAs must finish before TMEM is released.
      if (issued) {
        mma_commit(&bars->drain);
        volatile int32_t no_abort = 0;
        mbar_wait(&bars->drain, 0, &no_abort, p.status, kDevTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroup
    const int row = threadIdx.x;  // 0..127, TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const float scale_log2 = p.scale * kLog2e;  // > 0 (checked on the host)
    uint32_t k_iter = 0;
    uint32_t g = 0;  // global index of the key tile being processed (S/P buffer g & 1)
    // Waits until the PV MMA of global tile t (buffer t & 1) has completed.
    auto wait_pv = [&](uint32_t t) -> bool {
      return mbar_wait(&bars->pv_done[t & 1], (t >> 1) & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns);
    };
    bool ok = true;
    // SLOT_FIELDS inputs of a work item are fetched one item ahead: the pose
    // row into w and (sf_vec4) the head's slot values into shared memory,
    // issued after the previous item's last score tile so that they land
    // while its epilogue waits for the last PV.  sf_ready: the 4 warps staged
    // item c's slot values; sf_free: the 4 warps built item c's table (the
    // staging area may be overwritten).  c counts this CTA's items.
    float w[kMaxPoses];
    uint32_t sf_count = 0;
    auto sf_begin = [&](uint32_t it) -> bool {
      const uint32_t ibh = it / n_qt;
      load_pose_row(w, a, ibh / H, ibh % H, static_cast<int64_t>(it % n_qt) * BM + row);
      if (!a.sf_vec4) return true;
      if (sf_count > 0 &&
          !mbar_wait(&bars->sf_free, (sf_count - 1) & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns))
        return false;
      stage_slot_fields(table_s + a.sf_offset, a, ibh % H, row, BM);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->sf_ready);
      return true;
    };
    auto sf_finish = [&](int64_t head) -> bool {
      if (a.sf_vec4 && !mbar_wait(&bars->sf_ready, sf_count & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns))
        return false;
      build_table_sf(table_s, table_s + a.sf_offset, a, head, row, w);
      if (a.sf_vec4) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->sf_free);
      }
      ++sf_count;
      return true;
    };
    if (use_bias && a.slot_fields && blockIdx.x < n_items) ok = sf_begin(blockIdx.x);
    for (uint32_t item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const uint32_t qt = item % n_qt;
      const uint32_t bh = item / n_qt;
      const int64_t h = bh % H, b = bh / H;
      const int64_t i = static_cast<int64_t>(qt) * BM + row;  // token index of this thread's row
      // Flags of the item's first 64 key tiles, loaded before the table so
      // that the two memory round trips overlap.
      uint8_t fl0 = 0, fl1 = 0;
      if (use_bias) {
        fl0 = lane < n_kt ? p.slot_tile_flags[qt * n_kt + lane] : 0;
        fl1 = lane + 32 < n_kt ? p.slot_tile_flags[qt * n_kt + lane + 32] : 0;
        if (a.slot_fields) {
          if (!sf_finish(h)) {
            ok = false;
            break;
          }
        } else {
          stage_table(table_s, a, b, h, i, row);
          const uint32_t next = item + gridDim.x;
          if (next < n_items) {
            const uint32_t nbh = next / n_qt;
            prefetch_table_row(a, nbh / H, nbh % H, static_cast<int64_t>(next % n_qt) * BM + row);
          }
        }
      }
      float m = -INFINITY;
      uint64_t tile_mask = 0;  // bit k: key tile (j & ~63) + k carries Look bias for this warp
      for (int64_t j = 0; j < n_kt; ++j, ++k_iter) {
        if (use_bias && (j & 63) == 0) {
          // Each warp gathers the flags of the next 64 key tiles with one ballot pair.
          if (j > 0) {
            const int64_t t0 = j + lane, t1 = j + 32 + lane;
            fl0 = t0 < n_kt ? p.slot_tile_flags[qt * n_kt + t0] : 0;
            fl1 = t1 < n_kt ? p.slot_tile_flags[qt * n_kt + t1] : 0;
          }
          tile_mask = static_cast<uint64_t>(__ballot_sync(0xffffffffu, (fl0 >> warp) & 1)) |
                      (static_cast<uint64_t>(__ballot_sync(0xffffffffu, (fl1 >> warp) & 1)) << 32);
        }
        const uint32_t sb = g & 1;
        if (!mbar_wait(&bars->s_full[sb], (g >> 1) & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t s_addr = lane_base + (sb ? kColS1 : kColS0);
        float2 t[BN / 2];  // t[c] holds keys 2c and 2c+1
        load_s_row(s_addr, t);

        // t holds raw scores on tiles without Look bias, and the log2-domain
        // logits scale*log2(e)*s + bias on tiles with it.
        const uint32_t st = k_iter % KS;
        const bool bias_tile = (tile_mask >> (j & 63)) & 1u;
        if (bias_tile) {
          if (!mbar_wait(&bars->k_full[st], (k_iter / KS) & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns)) {
            ok = false;
            break;
          }
          add_look_bias(t, slot_s + st * kSlotBytes + row * 16, table_s + row, scale_log2);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->k_empty[st]);

        // Keys past the sequence end: the slot path looks them up as -inf (the
        // packed table marks them); without a Look bias mask them here.
        if (!use_bias) {
          const int32_t valid = static_cast<int32_t>(N - j * BN < BN ? N - j * BN : BN);
          if (valid < BN) {
#pragma unroll
            for (int c = 0; c < BN / 2; ++c) {
              if (2 * c >= valid) t[c].x = -INFINITY;
              if (2 * c + 1 >= valid) t[c].y = -INFINITY;
            }
          }
        }
        float mx = row_max64(t);
        if (!bias_tile) mx *= scale_log2;

        if (j == 0) {
          m = mx;
        } else {
          const bool need = mx > m + kRescaleThreshold;
          if (__any_sync(0xffffffffu, need)) {
            // O is read-modify-written: every PV issued so far (up to tile g-1) must be done.
            if (!wait_pv(g - 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const float f = need ? fast_exp2(m - mx) : 1.f;
            uint32_t r[16];
#pragma unroll
            for (int c = 0; c < ON / 16; ++c) {
              tmem_ld16(lane_base + kColO + c * 16, r);
              tmem_wait_ld();
              reg_fence16(r);
#pragma unroll
              for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * f);
              tmem_st16(lane_base + kColO + c * 16, r);
            }
            if (need) m = mx;
          }
        }
        // Probabilities (log2 domain, relative to the running max), written as
        // 16-bit pairs over the S columns they came from.  The row sum is not
        // kept here: the PV MMA accumulates it into O column 64.
        uint32_t w[BN / 2];
        exp_pack<BF16>(t, bias_tile ? 1.f : scale_log2, m, w);
        tmem_st16(s_addr, *reinterpret_cast<const uint32_t(*)[16]>(w));
        tmem_st16(s_addr + 16, *reinterpret_cast<const uint32_t(*)[16]>(w + 16));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[g & 1]);
        ++g;
      }
      if (!ok) break;
      if (use_bias && a.slot_fields && item + gridDim.x < n_items && !sf_begin(item + gridDim.x)) {
        ok = false;
        break;
      }
      // Epilogue: wait for the item's last PV, normalise by the row sum (O column 64), store.
      if (!wait_pv(g - 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t packed[HD / 2];
      float l;
      {
        uint32_t r0[16], r1[16], r2[16], r3[16], r4[16];
        tmem_ld16(lane_base + kColO, r0);
        tmem_ld16(lane_base + kColO + 16, r1);
        tmem_ld16(lane_base + kColO + 32, r2);
        tmem_ld16(lane_base + kColO + 48, r3);
        tmem_ld16(lane_base + kColO + 64, r4);
        tmem_wait_ld();
        reg_fence16(r0);
        reg_fence16(r1);
        reg_fence16(r2);
        reg_fence16(r3);
        reg_fence16(r4);
        l = __uint_as_float(r4[0]);
        const float inv = 1.f / l;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          packed[e] = pack_out<BF16>(r0[2 * e], r0[2 * e + 1], inv);
          packed[8 + e] = pack_out<BF16>(r1[2 * e], r1[2 * e + 1], inv);
          packed[16 + e] = pack_out<BF16>(r2[2 * e], r2[2 * e + 1], inv);
          packed[24 + e] = pack_out<BF16>(r3[2 * e], r3[2 * e + 1], inv);
        }
      }
      tc_fence_before();
      if (i < N) {
        uint8_t* dst = static_cast<uint8_t*>(p.out) +
                       2 * (b * p.out_stride[0] + h * p.out_stride[1] + i * p.out_stride[2]);
#pragma unroll
        for (int c = 0; c < HD / 8; ++c)
          reinterpret_cast<uint4*>(dst)[c] =
              make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
        if (p.lse != nullptr) p.lse[(b * H + h) * N + i] = (m + __log2f(l)) * kLn2;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
uint32_t table_bytes_for(int32_t n_slots) {
  return n_slots > 0 ? static_cast<uint32_t>((n_slots + 2) * BM * sizeof(float)) : 0u;
}

template <int KS>
size_t smem_bytes_for(uint32_t table_bytes) {
  size_t bytes = 1024 + SmemLayout<KS>::table + table_bytes + sizeof(Barriers<KS>) + 64;
  // Keep at most two CTAs per SM so two TMEM allocations of 256 columns fit.
  const size_t floor_bytes = 80 * 1024;
  return bytes < floor_bytes ? floor_bytes : bytes;
}

// Sets the kernel's shared-memory attributes, works out how many CTAs fit on
// an SM (at most two: two 256-column TMEM allocations) and launches a
// persistent grid of that many CTAs per SM.
template <int KS, bool BF16>
int32_t launch_variant(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const TcArgs& a,
                       size_t smem, int smem_per_sm, int regs_per_sm, int sm_count, cudaStream_t stream) {
  auto kernel = sla_tc_kernel<KS, BF16>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
          cudaSuccess ||
      cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
          cudaSuccess)
    return 6;
  // Resident CTAs per SM from the register and shared-memory budgets (the
  // occupancy query does not account for the carveout set above).
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess) return 6;
  const int warp_regs = ((fa.numRegs * 32 + 255) / 256) * 256;
  const int by_regs = regs_per_sm / (warp_regs * (kThreads / 32));
  const int by_smem = smem_per_sm / static_cast<int>(smem + 1024);
  int per_sm = by_regs < by_smem ? by_regs : by_smem;
  if (per_sm > 2) per_sm = 2;
  if (per_sm < 1) return 6;
  int64_t grid = static_cast<int64_t>(sm_count) * per_sm;
  if (grid > a.n_items) grid = a.n_items;
  kernel<<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(mq, mk, mv, a);
  return cudaGetLastError() == cudaSuccess ? 0 : 6;
}

}  // namespace

// What both tensor-core kernels need: 16-bit q / k / v / out with head_dim 64
// in layouts TMA can read, a status word, sane sizes and scale.
int32_t tc_common_ok(const SlaParams& p) {
  if (p.dtype != 1 && p.dtype != 2) return 0;
  if (p.head_dim != HD) return 0;
  if (p.status == nullptr) return 0;
  if (p.seq < 2 || p.seq > (int64_t(1) << 30) || p.batch > (int64_t(1) << 30) || p.heads > (int64_t(1) << 30))
    return 0;
  if (p.batch * p.heads * ((p.seq + BM - 1) / BM) > INT32_MAX) return 0;  // 32-bit work-item indices
  if (!(p.scale > 0.f) || !(p.scale < 3.0e38f)) return 0;
  if (!tma_stride_ok(p.q, p.q_stride) || !tma_stride_ok(p.k, p.k_stride) || !tma_stride_ok(p.v, p.v_stride))
    return 0;
  if (reinterpret_cast<uintptr_t>(p.out) % 16 || p.out_stride[3] != 1) return 0;
  for (int d = 0; d < 3; ++d)
    if ((p.out_stride[d] * 2) % 16) return 0;
  if (!get_encode_fn()) return 0;
  return 1;
}

// The tiled kernel (any N): no bias, SLOTS or SLOT_FIELDS, no dense bias.
int32_t sla_long_supported(const SlaParams& p) {
  if (!tc_common_ok(p)) return 0;
  if (p.dense != nullptr) return 0;
  if (p.bias_mode != 0 && p.bias_mode != 2 && p.bias_mode != 3) return 0;
  if (p.bias_mode == 2 && (p.poses < 1 || p.poses > kMaxSlots || !p.slots_packed || !p.slot_tile_flags)) return 0;
  if (p.bias_mode == 3 && (p.slots < 1 || p.slots > kMaxSlots || p.poses < 1 || p.poses > kMaxPoses ||
                           !p.slots_packed || !p.slot_tile_flags || !p.fields))
    return 0;
  return 1;
}

int32_t sla_tc_supported(const SlaParams& p) { return sla_short_supported(p) || sla_long_supported(p) ? 1 : 0; }

int32_t launch_sla_tc(const SlaParams& p, cudaStream_t stream, int sm_count) {
  if (sla_short_supported(p)) return launch_sla_short(p, stream, sm_count);  // N <= 256: one pass per row
  if (!sla_long_supported(p)) return 8;
  CUtensorMap mq, mk, mv;
  TcArgs a;
  if (!make_map(&mq, &a.oq, p.q, p.q_stride, p, BM) || !make_map(&mk, &a.ok, p.k, p.k_stride, p, BN) ||
      !make_map(&mv, &a.ov, p.v, p.v_stride, p, BN))
    return 4;
  a.p = p;
  a.wait_ns = tc_wait_budget_ns();
  a.n_qt = (p.seq + BM - 1) / BM;
  a.n_kt = (p.seq + BN - 1) / BN;
  a.n_items = p.batch * p.heads * a.n_qt;
  a.n_slots = p.bias_mode == 2 ? static_cast<int32_t>(p.poses) : (p.bias_mode == 3 ? static_cast<int32_t>(p.slots) : 0);
  a.slot_fields = p.bias_mode == 3 ? 1 : 0;
  a.n_poses = p.bias_mode == 3 ? static_cast<int32_t>(p.poses) : 0;
  a.sf_vec4 = 0;
  if (p.bias_mode == 3 && p.fields_dtype == 0 && p.fields_stride[2] == 1 && a.n_slots % 4 == 0 &&
      reinterpret_cast<uintptr_t>(p.fields) % 16 == 0 && p.fields_stride[0] % 4 == 0 && p.fields_stride[1] % 4 == 0)
    a.sf_vec4 = 1;
  a.table_bytes = table_bytes_for(a.n_slots);
  a.sf_offset = 0;
  if (a.sf_vec4) {  // staged slot values after the table rows: P x S fp32
    a.sf_offset = a.table_bytes / 4;
    a.table_bytes += static_cast<uint32_t>(a.n_poses * a.n_slots * 4);
  }
  a.pose_vec4 = 0;
  if (p.bias_mode == 3 && p.pose_dtype == 0 && p.pose_stride[3] == 1 && a.n_poses % 4 == 0 &&
      reinterpret_cast<uintptr_t>(p.pose) % 16 == 0 && p.pose_stride[0] % 4 == 0 && p.pose_stride[1] % 4 == 0 &&
      p.pose_stride[2] % 4 == 0)
    a.pose_vec4 = 1;
  if (p.bias_mode == 2 && p.pose_dtype == 0 && p.pose_stride[3] == 1 && a.n_slots % 4 == 0 &&
      reinterpret_cast<uintptr_t>(p.pose) % 16 == 0 && p.pose_stride[0] % 4 == 0 && p.pose_stride[1] % 4 == 0 &&
      p.pose_stride[2] % 4 == 0)
    a.pose_vec4 = 1;
  int dev = 0, smem_per_sm = 0, regs_per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&regs_per_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev) != cudaSuccess)
    return 6;
  const bool bf16 = p.dtype == 2;
  // Three K / slot-tile stages when two CTAs still fit on an SM, else two.
  const size_t smem3 = smem_bytes_for<3>(a.table_bytes), smem2 = smem_bytes_for<2>(a.table_bytes);
  const bool three = 2 * (smem3 + 1024) <= static_cast<size_t>(smem_per_sm);
  if (three)
    return bf16 ? launch_variant<3, true>(mq, mk, mv, a, smem3, smem_per_sm, regs_per_sm, sm_count, stream)
                : launch_variant<3, false>(mq, mk, mv, a, smem3, smem_per_sm, regs_per_sm, sm_count, stream);
  return bf16 ? launch_variant<2, true>(mq, mk, mv, a, smem2, smem_per_sm, regs_per_sm, sm_count, stream)
              : launch_variant<2, false>(mq, mk, mv, a, smem2, smem_per_sm, regs_per_sm, sm_count, stream);
}

}  // namespace intp
