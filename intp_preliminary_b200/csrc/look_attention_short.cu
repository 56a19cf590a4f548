// look_attention_short.cu - tcgen05 / TMA structured Look attention forward for
// sequences of at most 256 tokens (sm_100a).
//
// Semantics: layers/triton_structured_look_attention.py:25-54 (oracle) and
// :57-169 (the reference's Triton forward), for bf16 / f16 q, k, v with
// head_dim 64 and the Look bias in SLOTS form, SLOT_FIELDS form or none - the
// same coverage as look_attention_tc.cu, which handles every length.  The
// half6d3r model runs here (N = 196 tokens: CLS + 195 patches).
//
// At N <= 256 a whole score row fits in tensor memory, so there is no online
// softmax.  A work item is one (batch, head): its queries form at most two
// 128-row tiles A and B, and all N keys (rounded up to KR, a multiple of 16)
// form one tile.
//   * MMA: S_x = Q_x K^T (M = 128, N = KR, K = 64) for x = A, B, into TMEM
//     region x (R >= KR columns).  After the softmax, O_x = P_x V (K = KR,
//     N = 64) with P_x read from TMEM (16-bit pairs over the first KR/2
//     columns of the region) into the upper half of the same region.
//   * Softmax warpgroup x (one query row per thread = TMEM lane): pass 1 reads
//     S in 32-column chunks, adds the Look bias from the [slot][row] table
//     (log2 domain), keeps the row max and writes the logits back; pass 2
//     exponentiates relative to the exact row max, sums, and writes P and the
//     row's (max, sum) to TMEM.  While the PV MMA, the epilogue and the next
//     S MMA run, it builds its table for the next item.
//   * Look warpgroup: stages each item's slot values (SLOT_FIELDS) one item
//     ahead in a double buffer, and does the epilogue (O / l, 16-bit store,
//     LSE) off the softmax warps' path.
//   * Producer warp: the packed pair table once per CTA (resident for every
//     item: all items share the lattice), then per item Q_A, Q_B and K on one
//     barrier (reloaded once the S MMAs read them) and V on another.
// CTA: 512 threads (warps 0-3 softmax A, 4-7 softmax B, 8-11 Look, 12
// producer, 13 / 14 MMA issuers of tiles A / B (13 owns TMEM), 15 idle), one CTA per SM,
// persistent over (batch, head) items.  Every mbarrier wait is bounded; on
// expiry the CTA unwinds, drains its own copies and MMAs, frees TMEM and
// reports through the status word.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "sla_internal.h"
#include "sla_look_table.cuh"
#include "sla_tc_common.cuh"
#include "sm100_ptx.cuh"

namespace intp {
namespace {

constexpr int QM = 128;                       // query rows per tile
constexpr int SHD = 64;                       // head_dim
constexpr int kShortThreads = 512;
constexpr int kMaxShortSeq = 256;
constexpr int kMaxShortFieldPoses = 64;       // FIELDS: poses summed per key in pass 1
constexpr uint32_t kQTile = QM * SHD * 2;     // 16 KB
constexpr uint32_t kPackedTile = kSlotTileBytes;  // 8 KB packed pair tile (128 q x 64 k)

struct alignas(8) ShortBars {
  uint64_t slots_full;            // resident packed pair table landed
  uint64_t qk_full, qk_empty;     // Q_A, Q_B, K of an item / the S MMAs read them
  uint64_t v_full, v_empty;       // V of an item / the PV MMAs read it
  uint64_t s_full[2];             // S_x computed
  uint64_t p_full[2];             // P_x written, row max / sum published (4 softmax warps)
  uint64_t o_full[2];             // O_x computed
  uint64_t o_free[2];             // O_x read by the epilogue: region x may be overwritten (4 Look warps)
  uint64_t sf_ready[2];           // SLOT_FIELDS: an item's slot values staged in buffer b (4 Look warps)
  uint64_t p1_done[2];            // softmax x finished pass 1: its Look table may be rebuilt (4 warps)
  uint64_t tab_full[2];           // the Look warpgroup built table x for the next item (4 Look warps)
  uint64_t stagger;               // tile A finished its first pass 1 (4 softmax warps): tile B starts
  uint64_t drain[2];
  uint32_t tmem_base;
  int32_t abort;
};

struct ShortArgs {
  SlaParams p;
  MapOrder oq, ok, ov;
  int32_t n_items;        // batch * heads
  int32_t n_tiles;        // query tiles per item (1 or 2)
  int32_t kr;             // key columns computed: N rounded up to 16
  int32_t region;         // TMEM columns per tile: max(kr, 128)
  int32_t n_kt;           // 64-key tiles of the packed pair table
  int32_t n_slots;        // 0: no Look bias
  int32_t slot_fields, n_poses, pose_vec4, sf_vec4;
  int32_t fields_mode;    // FIELDS: the general (H, P, Np, Np) fields, summed per key in pass 1
  uint32_t off_k, off_v, off_slots, off_table, off_sf, off_bars;  // smem offsets
  uint32_t sf_floats;     // SLOT_FIELDS: floats of one staging buffer (n_poses * n_slots)
  uint32_t table_floats;  // per tile: (n_slots + 2) * 128
  uint64_t wait_ns;       // budget of the pipeline waits
};

__device__ __forceinline__ float fmax3s(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2s(float lo, float hi) {
  return BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

// 32 fp32 columns of this thread's TMEM lane (two x16 loads, one wait).
__device__ __forceinline__ void ld32(uint32_t addr, float2 (&t)[16]) {
  uint32_t r0[16], r1[16];
  tmem_ld16(addr, r0);
  tmem_ld16(addr + 16, r1);
  tmem_wait_ld();
  reg_fence16(r0);
  reg_fence16(r1);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    t[e] = make_float2(__uint_as_float(r0[2 * e]), __uint_as_float(r0[2 * e + 1]));
    t[8 + e] = make_float2(__uint_as_float(r1[2 * e]), __uint_as_float(r1[2 * e + 1]));
  }
}

__device__ __forceinline__ void st32(uint32_t addr, const float2 (&t)[16]) {
  uint32_t r0[16], r1[16];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    r0[2 * e] = __float_as_uint(t[e].x);
    r0[2 * e + 1] = __float_as_uint(t[e].y);
    r1[2 * e] = __float_as_uint(t[8 + e].x);
    r1[2 * e + 1] = __float_as_uint(t[8 + e].y);
  }
  tmem_st16(addr, r0);
  tmem_st16(addr + 16, r1);
}

// Pass 1 on one 32-key chunk (keys c0 .. c0+31): logits in the log2 domain,
// Look bias from the table through the 32 slot bytes `sb` of this row, and the
// running row max.  Columns past the last key (kr) are not touched by the
// caller; keys in [N, kr) carry the "past the end" slot (bias paths) or are
// masked here (no-bias path).
__device__ __forceinline__ float chunk_logits(float2 (&t)[16], float scale_log2, bool bias, const uint8_t* sb,
                                              const float* trow, bool mask, int32_t valid_keys, float m) {
  if (bias) {
    const uint4 w0 = *reinterpret_cast<const uint4*>(sb);
    const uint4 w1 = *reinterpret_cast<const uint4*>(sb + 2048);
    const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const uint32_t s0 = __byte_perm(ww[e >> 2], 0u, 0x4440u | (e & 3));
      const uint32_t s1 = __byte_perm(ww[e >> 2], 0u, 0x4440u | ((e + 1) & 3));
      float2& tv = t[e / 2];
      tv.x = fmaf(tv.x, scale_log2, trow[s0 * kTableRows]);
      tv.y = fmaf(tv.y, scale_log2, trow[s1 * kTableRows]);
    }
  } else {
    const float2 c2 = make_float2(scale_log2, scale_log2);
#pragma unroll
    for (int e = 0; e < 16; ++e) t[e] = mul2(t[e], c2);
    if (mask) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (2 * e >= valid_keys) t[e].x = -INFINITY;
        if (2 * e + 1 >= valid_keys) t[e].y = -INFINITY;
      }
    }
  }
  float m4[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2* v = t + 4 * k;
    m4[k] = fmaxf(fmax3s(fmax3s(v[0].x, v[0].y, v[1].x), fmax3s(v[1].y, v[2].x, v[2].y), v[3].x), v[3].y);
  }
  return fmax3s(fmax3s(m4[0], m4[1], m), m4[2], m4[3]);
}

// Running row max over a 32-key chunk of logits.
__device__ __forceinline__ float row_max32(const float2 (&t)[16], float m) {
  float m4[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2* v = t + 4 * k;
    m4[k] = fmaxf(fmax3s(fmax3s(v[0].x, v[0].y, v[1].x), fmax3s(v[1].y, v[2].x, v[2].y), v[3].x), v[3].y);
  }
  return fmax3s(fmax3s(m4[0], m4[1], m), m4[2], m4[3]);
}

// The general Look terms of the reference's form for query token i and key
// tokens c0 .. c0+nk-1 (log2 domain, added to t): the dense bias
// dense[b, h, i-1, j-1] and the FIELDS bias sum_p pose[b, i-1, h, p] *
// fields[h, p, i-1, j-1] (layers/triton_structured_look_attention.py:116-139);
// the CLS token (0) and keys past the sequence get neither.
template <class A>
__device__ __forceinline__ void add_general_bias(float2 (&t)[16], const A& a, uint32_t item, int32_t i, int c0,
                                                 int nk) {
  const SlaParams& p = a.p;
  const int32_t N = static_cast<int32_t>(p.seq);
  if (i < 1 || i >= N) return;
  const int64_t h = item % static_cast<uint32_t>(p.heads), b = item / static_cast<uint32_t>(p.heads);
  float add[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) add[e] = 0.f;
  if (p.dense != nullptr) {
    const int64_t base = b * p.dense_stride[0] + h * p.dense_stride[1] + (i - 1) * p.dense_stride[2];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int32_t j = c0 + e;
      if (e < nk && j >= 1 && j < N) add[e] = load_any(p.dense, base + (j - 1) * p.dense_stride[3], p.dense_dtype);
    }
  }
  if (a.fields_mode) {
    const int64_t pbase = b * p.pose_stride[0] + (i - 1) * p.pose_stride[1] + h * p.pose_stride[2];
    for (int pp = 0; pp < a.n_poses; ++pp) {
      const float w = load_any(p.pose, pbase + pp * p.pose_stride[3], p.pose_dtype);
      const int64_t fbase = h * p.fields_stride[0] + pp * p.fields_stride[1] + (i - 1) * p.fields_stride[2];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int32_t j = c0 + e;
        if (e < nk && j >= 1 && j < N)
          add[e] = fmaf(w, load_any(p.fields, fbase + (j - 1) * p.fields_stride[3], p.fields_dtype), add[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    t[e].x = fmaf(add[2 * e], kLog2eF, t[e].x);
    t[e].y = fmaf(add[2 * e + 1], kLog2eF, t[e].y);
  }
}

// GENERAL: the dense-bias / general-fields terms are compiled in (a separate
// instance, so the SLOTS / SLOT_FIELDS / no-bias path carries no code for them).
template <bool BF16, bool GENERAL>
__global__ void __launch_bounds__(kShortThreads, 1)
sla_short_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const ShortArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  ShortBars* bars = reinterpret_cast<ShortBars*>(smem + a.off_bars);
  uint8_t* q_s = smem;                      // Q_A, Q_B
  uint8_t* k_s = smem + a.off_k;
  uint8_t* v_s = smem + a.off_v;
  uint8_t* slots_s = smem + a.off_slots;
  float* table_s = reinterpret_cast<float*>(smem + a.off_table);  // tile x at x * table_floats
  float* sf_s = reinterpret_cast<float*>(smem + a.off_sf);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const SlaParams& p = a.p;
  volatile int32_t* abort_flag = &bars->abort;
  const bool use_bias = a.n_slots > 0;
  const int32_t N = static_cast<int32_t>(p.seq);
  const uint32_t H = static_cast<uint32_t>(p.heads);
  const uint32_t n_items = static_cast<uint32_t>(a.n_items);
  const int nt = a.n_tiles;

  if (threadIdx.x == 0) {
    mbar_init(&bars->slots_full, 1);
    mbar_init(&bars->qk_full, 1);
    mbar_init(&bars->qk_empty, nt);  // one commit per tile's S MMA
    mbar_init(&bars->v_full, 1);
    mbar_init(&bars->v_empty, nt);   // one commit per tile's PV MMA
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->s_full[x], 1);
      mbar_init(&bars->p_full[x], 4);
      mbar_init(&bars->o_full[x], 1);
      mbar_init(&bars->o_free[x], 4);
      mbar_init(&bars->sf_ready[x], 4);
      mbar_init(&bars->p1_done[x], 4);
      mbar_init(&bars->tab_full[x], 4);
    }
    mbar_init(&bars->stagger, 4);
    mbar_init(&bars->drain[0], 1);
    mbar_init(&bars->drain[1], 1);
    bars->abort = 0;
    mbar_fence_init();
  }
  if (warp == 13) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 12) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const uint32_t n_packed = static_cast<uint32_t>(nt * a.n_kt);
      if (use_bias) {
        mbar_arrive_expect_tx(&bars->slots_full, n_packed * kPackedTile);
        for (uint32_t t = 0; t < n_packed; ++t)
          bulk_load(slots_s + t * kPackedTile, p.slots_packed + t * kPackedTile, kPackedTile, &bars->slots_full);
      }
      const uint32_t q_bytes = static_cast<uint32_t>(nt) * kQTile;
      const uint32_t kv_bytes = static_cast<uint32_t>(a.kr) * 128u;
      uint32_t k = 0, qk_issued = 0, v_issued = 0;
      bool ok = true;
      for (uint32_t item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++k) {
        const int32_t h = static_cast<int32_t>(item % H), b = static_cast<int32_t>(item / H);
        if (k > 0 && !mbar_wait(&bars->qk_empty, (k - 1) & 1, abort_flag, p.status, kDevTimeoutProducer, a.wait_ns)) {
          ok = false;
          break;
        }
        ++qk_issued;
        mbar_arrive_expect_tx(&bars->qk_full, q_bytes + kv_bytes);
        for (int x = 0; x < nt; ++x) {
          const int32_t r = x * QM;
          tma_load_4d(q_s + x * kQTile, &tm_q, &bars->qk_full, 0, map_coord(a.oq, 1, r, h, b),
                      map_coord(a.oq, 2, r, h, b), map_coord(a.oq, 3, r, h, b));
        }
        tma_load_4d(k_s, &tm_k, &bars->qk_full, 0, map_coord(a.ok, 1, 0, h, b), map_coord(a.ok, 2, 0, h, b),
                    map_coord(a.ok, 3, 0, h, b));
        if (k > 0 && !mbar_wait(&bars->v_empty, (k - 1) & 1, abort_flag, p.status, kDevTimeoutProducer, a.wait_ns)) {
          ok = false;
          break;
        }
        ++v_issued;
        mbar_arrive_expect_tx(&bars->v_full, kv_bytes);
        tma_load_4d(v_s, &tm_v, &bars->v_full, 0, map_coord(a.ov, 1, 0, h, b), map_coord(a.ov, 2, 0, h, b),
                    map_coord(a.ov, 3, 0, h, b));
      }
      // Drain: no copy may still be in flight into shared memory of an exiting CTA.
      volatile int32_t no_abort = 0;
      if (use_bias) mbar_wait(&bars->slots_full, 0, &no_abort, p.status, kDevTimeoutDrain);
      if (qk_issued > 0) mbar_wait(&bars->qk_full, (qk_issued - 1) & 1, &no_abort, p.status, kDevTimeoutDrain);
      if (v_issued > 0) mbar_wait(&bars->v_full, (v_issued - 1) & 1, &no_abort, p.status, kDevTimeoutDrain);
    }
  } else if (warp == 13 || warp == 14) {
    // ------------------------------------------------------------ MMA issuers
    // One issuing thread per query tile (warp 13: A, warp 14: B), so that the
    // two tiles' chains (S -> softmax -> PV -> epilogue) run independently and
    // tile B's lags tile A's by about one softmax pass: while one warpgroup
    // exponentiates (MUFU), the other adds the Look bias or builds its table.
    const int x = warp - 13;
    if (lane == 0 && x < nt) {
      const uint32_t idesc_s = idesc_f16(BF16, false, QM, static_cast<uint32_t>(a.kr));
      const uint32_t idesc_o = idesc_f16(BF16, true, QM, SHD);
      const uint64_t k_desc = smem_desc_sw128(smem_u32(k_s), 16, 1024);
      const uint64_t v_desc = smem_desc_sw128(smem_u32(v_s), static_cast<uint32_t>(a.kr) * 128u, 1024);
      const uint64_t q_desc = smem_desc_sw128(smem_u32(q_s + x * kQTile), 16, 1024);
      const uint32_t R = static_cast<uint32_t>(a.region);
      const uint32_t s_col = tmem + x * R, o_col = tmem + x * R + R / 2;
      const int ksteps = a.kr / 16;
      uint32_t k = 0;
      bool ok = true, issued = false;
      if (x == 1 && blockIdx.x < n_items)
        ok = mbar_wait(&bars->stagger, 0, abort_flag, p.status, kDevTimeoutMma, a.wait_ns);
      for (uint32_t item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++k) {
        if (!mbar_wait(&bars->qk_full, k & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) {
          ok = false;
          break;
        }
        // Region x holds the previous item's P_x and O_x until its epilogue read O_x.
        if (k > 0 && !mbar_wait(&bars->o_free[x], (k - 1) & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < SHD / 16; ++kk)
          mma_ss(s_col, q_desc + ((kk * 32) >> 4), k_desc + ((kk * 32) >> 4), idesc_s, kk > 0 ? 1u : 0u);
        mma_commit(&bars->s_full[x]);
        mma_commit(&bars->qk_empty);
        issued = true;
        if (!mbar_wait(&bars->v_full, k & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns) ||
            !mbar_wait(&bars->p_full[x], k & 1, abort_flag, p.status, kDevTimeoutMma, a.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kk = 0; kk < ksteps; ++kk)
          mma_ts(o_col, s_col + kk * 8, v_desc + ((kk * 2048) >> 4), idesc_o, kk > 0 ? 1u : 0u);
        mma_commit(&bars->o_full[x]);
        mma_commit(&bars->v_empty);
      }
      if (issued) {
        mma_commit(&bars->drain[x]);
        volatile int32_t no_abort = 0;
        mbar_wait(&bars->drain[x], 0, &no_abort, p.status, kDevTimeoutDrain);
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax warpgroups
    const int x = warp >> 2;                       // query tile A (0) or B (1)
    const int qw = warp & 3;                       // TMEM lane quadrant
    const int row = qw * 32 + lane;                // row within the tile = TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(qw * 32) << 16) + x * static_cast<uint32_t>(a.region);
    const float scale_log2 = p.scale * kLog2eF;
    const int32_t tok = x * QM + row;
    const bool warp_live = x < nt && x * QM + qw * 32 < N;  // some row of this warp is a token
    constexpr bool general = GENERAL;
    float* trow = table_s + x * a.table_floats + row;
    const uint8_t* srow = slots_s + static_cast<uint32_t>(x * a.n_kt) * kPackedTile + row * 16;
    // Per 64-key tile of the pair table: does this warp's block carry Look bias
    // (or padding keys)?  The same for every item.
    uint32_t bias_tiles = 0;
    if (use_bias && x < nt)
      for (int kt = 0; kt < a.n_kt; ++kt)
        if ((p.slot_tile_flags[x * a.n_kt + kt] >> qw) & 1) bias_tiles |= 1u << kt;
    bool ok = x < nt;
    if (ok && use_bias) ok = mbar_wait(&bars->slots_full, 0, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns);
    uint32_t k = 0;
    for (uint32_t item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++k) {
      // The item's Look table, built by the Look warpgroup while this
      // warpgroup ran pass 2 of the previous item.
      if (use_bias && !mbar_wait(&bars->tab_full[x], k & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns)) {
        ok = false;
        break;
      }
      if (!mbar_wait(&bars->s_full[x], k & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float m = -INFINITY, l = 0.f;
      if (warp_live) {
        // pass 1: logits (log2 domain, Look bias added) and the row max
        for (int c0 = 0; c0 < a.kr; c0 += 32) {
          float2 t[16];
          const bool half = c0 + 32 > a.kr;  // a 16-column tail
          if (half) {
            uint32_t r0[16];
            tmem_ld16(lane_base + c0, r0);
            tmem_wait_ld();
            reg_fence16(r0);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              t[e] = make_float2(__uint_as_float(r0[2 * e]), __uint_as_float(r0[2 * e + 1]));
              t[8 + e] = make_float2(-INFINITY, -INFINITY);
            }
          } else {
            ld32(lane_base + c0, t);
          }
          if constexpr (!general) {
          const int kt = c0 >> 6;
          const bool bias = (bias_tiles >> kt) & 1u;
          const uint8_t* sb = srow + kt * kPackedTile + ((c0 & 63) >> 4) * 2048;
          if (bias && half) {
            // a 16-key tail with bias: the second 16 bytes are not ours to read
            const uint4 w0 = *reinterpret_cast<const uint4*>(sb);
            const uint32_t ww[4] = {w0.x, w0.y, w0.z, w0.w};
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const uint32_t s0 = __byte_perm(ww[e >> 2], 0u, 0x4440u | (e & 3));
              const uint32_t s1 = __byte_perm(ww[e >> 2], 0u, 0x4440u | ((e + 1) & 3));
              t[e / 2].x = fmaf(t[e / 2].x, scale_log2, trow[s0 * kTableRows]);
              t[e / 2].y = fmaf(t[e / 2].y, scale_log2, trow[s1 * kTableRows]);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) m = fmax3s(m, t[e].x, t[e].y);
          } else {
            m = chunk_logits(t, scale_log2, bias, sb, trow, !use_bias && c0 + 32 > N, N - c0, m);
          }
          } else {
          const int kt = c0 >> 6;
          const bool bias = (bias_tiles >> kt) & 1u;
          const uint8_t* sb = srow + kt * kPackedTile + ((c0 & 63) >> 4) * 2048;
          if (bias) {
            // logits = scale log2(e) s + table[slot]; a 16-key tail reads 16 slot bytes
            const uint4 w0 = *reinterpret_cast<const uint4*>(sb);
            const uint4 w1 = half ? make_uint4(0u, 0u, 0u, 0u) : *reinterpret_cast<const uint4*>(sb + 2048);
            const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const uint32_t s0 = __byte_perm(ww[e >> 2], 0u, 0x4440u | (e & 3));
              const uint32_t s1 = __byte_perm(ww[e >> 2], 0u, 0x4440u | ((e + 1) & 3));
              t[e / 2].x = fmaf(t[e / 2].x, scale_log2, trow[s0 * kTableRows]);
              t[e / 2].y = fmaf(t[e / 2].y, scale_log2, trow[s1 * kTableRows]);
            }
          } else {
            const float2 c2 = make_float2(scale_log2, scale_log2);
#pragma unroll
            for (int e = 0; e < 16; ++e) t[e] = mul2(t[e], c2);
          }
          if constexpr (general) add_general_bias(t, a, item, tok, c0, half ? 16 : 32);
          if (!use_bias && c0 + 32 > N) {
            // no pair table marks the keys past the end: mask them here
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              if (c0 + 2 * e >= N) t[e].x = -INFINITY;
              if (c0 + 2 * e + 1 >= N) t[e].y = -INFINITY;
            }
          }
          if (half) {
#pragma unroll
            for (int e = 8; e < 16; ++e) t[e] = make_float2(-INFINITY, -INFINITY);
          }
          m = row_max32(t, m);
          }
          if (half) {
            uint32_t r0[16];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              r0[2 * e] = __float_as_uint(t[e].x);
              r0[2 * e + 1] = __float_as_uint(t[e].y);
            }
            tmem_st16(lane_base + c0, r0);
          } else {
            st32(lane_base + c0, t);
          }
        }
        tmem_wait_st();
      }
      __syncwarp();
      if (lane == 0) {
        if (use_bias) mbar_arrive(&bars->p1_done[x]);  // table reads of this item are done
        if (x == 0 && k == 0 && nt == 2) mbar_arrive(&bars->stagger);
      }
      if (warp_live) {
        // pass 2: P = 2^(logit - m), row sum, 16-bit pairs over the first kr/2 columns
        const float2 nm2 = make_float2(-m, -m), one2 = make_float2(1.f, 1.f);
        float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
        for (int c0 = 0; c0 < a.kr; c0 += 32) {
          float2 t[16];
          const bool half = c0 + 32 > a.kr;
          if (half) {
            uint32_t r0[16];
            tmem_ld16(lane_base + c0, r0);
            tmem_wait_ld();
            reg_fence16(r0);
#pragma unroll
            for (int e = 0; e < 8; ++e) t[e] = make_float2(__uint_as_float(r0[2 * e]), __uint_as_float(r0[2 * e + 1]));
#pragma unroll
            for (int e = 8; e < 16; ++e) t[e] = make_float2(-INFINITY, -INFINITY);
          } else {
            ld32(lane_base + c0, t);
          }
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float2 xx = fma2(t[e], one2, nm2);
            // a quarter of the pairs on the FMA pipe (exp2_fma), the rest on the MUFU
            const float2 pe = (e & 3) == 3 ? exp2_fma(xx) : make_float2(fast_exp2(xx.x), fast_exp2(xx.y));
            if (e & 1)
              acc1 = add2(acc1, pe);
            else
              acc0 = add2(acc0, pe);
            w[e] = pack2s<BF16>(pe.x, pe.y);
          }
          if (half) {
            uint32_t w8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) w8[e] = w[e];
            tmem_st8(lane_base + c0 / 2, w8);
          } else {
            tmem_st16(lane_base + c0 / 2, w);
          }
        }
        tmem_wait_st();
        l = (acc0.x + acc1.x) + (acc0.y + acc1.y);
      }
      {
        // (row max, row sum) next to O for the epilogue: columns R/2 + 64, + 65
        const uint32_t ml[2] = {__float_as_uint(m), __float_as_uint(l)};
        tmem_st2(lane_base + a.region / 2 + SHD, ml);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[x]);
    }
  } else if (warp < 12) {
    // ------------------------------------------------------------ Look warpgroup
    const int lt = threadIdx.x - 256;              // 0..127: row of both tiles
    const int qw = warp & 3;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(qw * 32) << 16);
    const uint32_t R = static_cast<uint32_t>(a.region);
    bool ok = true;
    // The epilogue of item `kk` (tile x): O / l, 16-bit store, LSE.
    auto epilogue = [&](uint32_t kk, uint32_t item, int x) -> bool {
      // p_full orders the softmax's (max, sum) store before this thread's load.
      if (!mbar_wait(&bars->p_full[x], kk & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns)) return false;
      if (!mbar_wait(&bars->o_full[x], kk & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns)) return false;
      tc_fence_after();
      uint32_t r0[16], r1[16], r2[16], r3[16], ml[2];
      const uint32_t o = lane_base + x * R + R / 2;
      tmem_ld16(o, r0);
      tmem_ld16(o + 16, r1);
      tmem_ld16(o + 32, r2);
      tmem_ld16(o + 48, r3);
      tmem_ld2(o + SHD, ml);
      tmem_wait_ld();
      reg_fence16(r0);
      reg_fence16(r1);
      reg_fence16(r2);
      reg_fence16(r3);
      asm volatile("" : "+r"(ml[0]), "+r"(ml[1])::"memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->o_free[x]);
      const int32_t i = x * QM + lt;
      if (i < N) {
        const float mx = __uint_as_float(ml[0]), l = __uint_as_float(ml[1]);
        const float inv = 1.f / l;
        const int64_t h = item % H, b = item / H;
        uint32_t packed[SHD / 2];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          packed[e] = pack2s<BF16>(__uint_as_float(r0[2 * e]) * inv, __uint_as_float(r0[2 * e + 1]) * inv);
          packed[8 + e] = pack2s<BF16>(__uint_as_float(r1[2 * e]) * inv, __uint_as_float(r1[2 * e + 1]) * inv);
          packed[16 + e] = pack2s<BF16>(__uint_as_float(r2[2 * e]) * inv, __uint_as_float(r2[2 * e + 1]) * inv);
          packed[24 + e] = pack2s<BF16>(__uint_as_float(r3[2 * e]) * inv, __uint_as_float(r3[2 * e + 1]) * inv);
        }
        uint8_t* dst = static_cast<uint8_t*>(p.out) + 2 * (b * p.out_stride[0] + h * p.out_stride[1] + i * p.out_stride[2]);
#pragma unroll
        for (int c = 0; c < SHD / 8; ++c)
          reinterpret_cast<uint4*>(dst)[c] =
              make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
        if (p.lse != nullptr) p.lse[(b * H + h) * N + i] = (mx + __log2f(l)) * 0.6931471805599453f;
      }
      return true;
    };
    // Slot values (SLOT_FIELDS) of the CTA's kk-th item into buffer kk & 1.
    // Its previous contents (item kk - 2) were read by this warpgroup's own
    // table builds for that item, which every Look warp finished before the
    // softmax could start that item's pass 1 (tab_full) - long before any Look
    // warp gets here, past the epilogues of item kk - 2.
    const bool stage = use_bias && a.slot_fields && a.sf_vec4;
    auto stage_sf = [&](uint32_t kk, uint32_t it) {
      stage_slot_fields(sf_s + (kk & 1) * a.sf_floats, a, it % H, lt, QM);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->sf_ready[kk & 1]);
    };
    // Table x of the CTA's kk-th item (`it`): SLOTS copies the rows' Look
    // values, SLOT_FIELDS forms pose x slot values (each warp its 32 rows,
    // the rows softmax warp qw of tile x reads).
    // SLOT_FIELDS: the pose rows of the next item's two tiles, loaded at the
    // top of an iteration so their memory latency passes while this warpgroup
    // waits for the softmax; `build` consumes them.
    auto build = [&](int x, uint32_t kk, uint32_t it) -> bool {
      const uint32_t h = it % H, b = it / H;
      const int32_t tok = x * QM + lt;
      float* tab = table_s + x * a.table_floats;
      if (!a.slot_fields) {
        stage_table(tab, a, b, h, tok, lt);
      } else {
        float w[kMaxLookPoses];
        load_pose_row(w, a, b, h, tok);
        if (a.sf_vec4 && !mbar_wait(&bars->sf_ready[kk & 1], (kk >> 1) & 1, abort_flag, p.status,
                                    kDevTimeoutSoftmax, a.wait_ns))
          return false;
        build_table_sf(tab, sf_s + (kk & 1) * a.sf_floats, a, h, lt, w);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tab_full[x]);
      return true;
    };
    uint32_t k = 0;
    if (use_bias && blockIdx.x < n_items) {
      if (stage) stage_sf(0, blockIdx.x);
      for (int x = 0; x < nt && ok; ++x) ok = build(x, 0, blockIdx.x);
    }
    for (uint32_t item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++k) {
      const uint32_t next = item + gridDim.x;
      if (stage && next < n_items) stage_sf(k + 1, next);
      for (int x = 0; x < nt && ok; ++x) {
        // Table x of the next item once softmax x is through pass 1 of this one
        // (it runs pass 2, the PV MMA and this epilogue meanwhile).
        if (use_bias && next < n_items) {
          if (!mbar_wait(&bars->p1_done[x], k & 1, abort_flag, p.status, kDevTimeoutSoftmax, a.wait_ns) ||
              !build(x, k + 1, next)) {
            ok = false;
            break;
          }
        }
        ok = epilogue(k, item, x);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

}  // namespace

int32_t sla_short_supported(const SlaParams& p) {
  if (p.seq < 2 || p.seq > kMaxShortSeq) return 0;
  if (!tc_common_ok(p)) return 0;
  switch (p.bias_mode) {
    case 0: break;
    case 1:
      if (!p.pose || !p.fields || p.poses < 1 || p.poses > kMaxShortFieldPoses) return 0;
      break;
    case 2:
      if (p.poses < 1 || p.poses > kMaxLookSlots || !p.slots_packed || !p.slot_tile_flags) return 0;
      break;
    case 3:
      if (p.slots < 1 || p.slots > kMaxLookSlots || p.poses < 1 || p.poses > kMaxLookPoses || !p.slots_packed ||
          !p.slot_tile_flags || !p.fields)
        return 0;
      break;
    default: return 0;
  }
  const int32_t n_slots =
      p.bias_mode == 2 ? static_cast<int32_t>(p.poses) : (p.bias_mode == 3 ? static_cast<int32_t>(p.slots) : 0);
  const int64_t kr = (p.seq + 15) / 16 * 16;
  if ((kr < 144 ? 144 : kr) * 2 > 512) return 0;  // two TMEM regions
  const int64_t n_tiles = (p.seq + QM - 1) / QM;
  const int64_t n_kt = (p.seq + kSlotTileK - 1) / kSlotTileK;
  int64_t bytes = 2 * kQTile + 2 * kr * 128;
  if (n_slots > 0) bytes += n_tiles * n_kt * kPackedTile + 2 * int64_t(n_slots + 2) * QM * 4;
  if (p.bias_mode == 3) bytes += 2 * int64_t(p.poses) * n_slots * 4;
  bytes += 512 + 1024;
  int dev = 0, optin = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return 0;
  return bytes <= optin ? 1 : 0;
}

int32_t launch_sla_short(const SlaParams& p, cudaStream_t stream, int sm_count) {
  if (!sla_short_supported(p)) return 8;
  ShortArgs a;
  a.p = p;
  a.kr = static_cast<int32_t>((p.seq + 15) / 16 * 16);
  a.region = a.kr < 144 ? 144 : a.kr;  // P below R/2, O at [R/2, R/2+64), (max, sum) at R/2+64
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, &a.oq, p.q, p.q_stride, p, QM) ||
      !make_map(&mk, &a.ok, p.k, p.k_stride, p, static_cast<uint32_t>(a.kr)) ||
      !make_map(&mv, &a.ov, p.v, p.v_stride, p, static_cast<uint32_t>(a.kr)))
    return 4;
  a.n_items = static_cast<int32_t>(p.batch * p.heads);
  a.n_tiles = static_cast<int32_t>((p.seq + QM - 1) / QM);
  a.n_kt = static_cast<int32_t>((p.seq + kSlotTileK - 1) / kSlotTileK);
  a.n_slots = p.bias_mode == 2 ? static_cast<int32_t>(p.poses) : (p.bias_mode == 3 ? static_cast<int32_t>(p.slots) : 0);
  a.slot_fields = p.bias_mode == 3 ? 1 : 0;
  a.fields_mode = p.bias_mode == 1 ? 1 : 0;
  a.n_poses = (p.bias_mode == 3 || p.bias_mode == 1) ? static_cast<int32_t>(p.poses) : 0;
  a.sf_vec4 = (p.bias_mode == 3 && p.fields_dtype == 0 && p.fields_stride[2] == 1 && a.n_slots % 4 == 0 &&
               reinterpret_cast<uintptr_t>(p.fields) % 16 == 0 && p.fields_stride[0] % 4 == 0 &&
               p.fields_stride[1] % 4 == 0)
                  ? 1 : 0;
  const int32_t vec_count = p.bias_mode == 3 ? a.n_poses : a.n_slots;
  a.pose_vec4 = ((p.bias_mode == 2 || p.bias_mode == 3) && p.pose_dtype == 0 && p.pose_stride[3] == 1 &&
                 vec_count % 4 == 0 && reinterpret_cast<uintptr_t>(p.pose) % 16 == 0 && p.pose_stride[0] % 4 == 0 &&
                 p.pose_stride[1] % 4 == 0 && p.pose_stride[2] % 4 == 0)
                    ? 1 : 0;
  a.table_floats = static_cast<uint32_t>(a.n_slots > 0 ? (a.n_slots + 2) * QM : 0);
  uint32_t off = 2 * kQTile;
  a.off_k = off;
  off = align_up(off + static_cast<uint32_t>(a.kr) * 128u, 1024);
  a.off_v = off;
  off = align_up(off + static_cast<uint32_t>(a.kr) * 128u, 1024);
  a.off_slots = off;
  if (a.n_slots > 0) off += static_cast<uint32_t>(a.n_tiles * a.n_kt) * kPackedTile;
  a.off_table = off;
  off += 2 * a.table_floats * 4;
  a.off_sf = off;
  a.sf_floats = a.slot_fields ? static_cast<uint32_t>(a.n_poses * a.n_slots) : 0u;
  off += 2 * a.sf_floats * 4;
  a.off_bars = align_up(off, 64);
  // At least half of an SM's shared memory: one CTA per SM, the only holder of
  // its 512 TMEM columns.
  size_t smem = a.off_bars + sizeof(ShortBars) + 1024;
  if (smem < 120 * 1024) smem = 120 * 1024;
  a.wait_ns = tc_wait_budget_ns();
  const bool general = a.fields_mode || p.dense != nullptr;
  auto kernel = p.dtype == 2 ? (general ? sla_short_kernel<true, true> : sla_short_kernel<true, false>)
                             : (general ? sla_short_kernel<false, true> : sla_short_kernel<false, false>);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return 6;
  int64_t grid = sm_count;
  if (grid > a.n_items) grid = a.n_items;
  kernel<<<static_cast<unsigned>(grid), kShortThreads, smem, stream>>>(mq, mk, mv, a);
  return cudaGetLastError() == cudaSuccess ? 0 : 6;
}

}  // namespace intp
