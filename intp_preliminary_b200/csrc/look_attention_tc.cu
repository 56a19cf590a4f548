// look_attention_tc.cu - tcgen05 / TMA structured Look attention forward (sm_100a).
//
// Semantics: layers/triton_structured_look_attention.py:25-54 (oracle) and
// :57-169 (the reference's Triton forward), for bf16 / f16 inputs, head_dim 64,
// with the Look bias in SLOTS form (bias[b,h,i,j] = pose[b,i-1,h,slot(i,j)],
// the one-hot-fields case of the reference API) or no bias.
//
// CTA organisation (192 threads, two CTAs per SM):
//   warps 0-3  softmax warpgroup: thread t owns query row t of the 128-row tile.
//              Reads S from TMEM, adds the Look bias from shared memory, runs the
//              online softmax in the log2 domain, writes P (16-bit) back to TMEM,
//              rescales O in TMEM when the running max grows by more than 2^8,
//              and finally normalises O and stores it (plus the LSE).
//   warp 4     TMA producer: Q tile (128 x 64) per work item, then K/V tiles of
//              64 keys plus the 8 KB packed slot tile, double buffered.
//   warp 5     MMA issuer: S = Q K^T (tcgen05.mma kind::f16, both operands in
//              shared memory, accumulator in TMEM) and O += P V (P from TMEM).
// TMEM columns: [0,64) S buffer 0, [64,128) S buffer 1, [128,192) O, [192,224) P.
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

namespace intp {
namespace {

constexpr int BM = 128;            // query rows per tile
constexpr int BN = 64;             // keys per tile
constexpr int HD = 64;             // head_dim
constexpr int kThreads = 192;
constexpr int kStages = 2;
constexpr uint32_t kQBytes = BM * HD * 2;      // 16 KB
constexpr uint32_t kKVBytes = BN * HD * 2;     // 8 KB each of K and V
constexpr uint32_t kSlotBytes = kSlotTileBytes;  // 8 KB
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS0 = 0, kColS1 = 64, kColO = 128, kColP = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P values stay <= 2^8
constexpr int kMaxSlots = 94;

struct alignas(8) Barriers {
  uint64_t q_full, q_empty;
  uint64_t kv_full[kStages], kv_empty[kStages];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full, pv_done;
  uint64_t drain;
  uint32_t tmem_base;
  int32_t abort;
};

struct SmemLayout {
  // offsets relative to a 1024-byte aligned base
  static constexpr uint32_t q = 0;
  static constexpr uint32_t k = q + kQBytes;
  static constexpr uint32_t v = k + kStages * kKVBytes;
  static constexpr uint32_t slots = v + kStages * kKVBytes;
  static constexpr uint32_t table = slots + kStages * kSlotBytes;
};

__device__ __forceinline__ float load_any(const void* p, int64_t idx, int32_t dtype) {
  switch (dtype) {
    case 1: return __half2float(static_cast<const __half*>(p)[idx]);
    case 2: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
    default: return static_cast<const float*>(p)[idx];
  }
}

// Position (1..3) of the row / head / batch coordinate in a tensor map whose
// outer dimensions are sorted by increasing stride (dimension 0 is head_dim).
struct MapOrder {
  int8_t row, head, batch;
};

// TMA coordinates {0, c1, c2, c3} with row / head / batch placed per `o`.
__device__ __forceinline__ int32_t map_coord(const MapOrder& o, int pos, int32_t row, int32_t head, int32_t batch) {
  return o.row == pos ? row : (o.head == pos ? head : batch);
}

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

__device__ __forceinline__ uint32_t pack_out(uint32_t lo, uint32_t hi, float inv, int32_t dtype) {
  const float a = __uint_as_float(lo) * inv, b = __uint_as_float(hi) * inv;
  return dtype == 2 ? pack_bf16x2(a, b) : pack_f16x2(a, b);
}

struct TcArgs {
  SlaParams p;
  MapOrder oq, ok, ov;
  int64_t n_qt, n_kt, n_items;
  int32_t n_slots;        // 0 when there is no Look bias
  uint32_t table_bytes;   // bytes of the per-query Look table in smem
  int32_t pose_vec4;      // pose rows are 16-byte aligned fp32 with unit slot stride
};

__global__ void __launch_bounds__(kThreads, 2)
sla_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + SmemLayout::table + a.table_bytes);
  uint8_t* q_s = smem + SmemLayout::q;
  uint8_t* k_s = smem + SmemLayout::k;
  uint8_t* v_s = smem + SmemLayout::v;
  uint8_t* slot_s = smem + SmemLayout::slots;
  float* table_s = reinterpret_cast<float*>(smem + SmemLayout::table);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const SlaParams& p = a.p;
  volatile int32_t* abort_flag = &bars->abort;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1 + 4);  // MMA commit + 4 softmax warps
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_free[s], 4);
    }
    mbar_init(&bars->p_full, 4);
    mbar_init(&bars->pv_done, 1);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    mbar_fence_init();
  }
  if (warp == 5) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  const int64_t N = p.seq;
  const int64_t H = p.heads;
  const int64_t n_kt = a.n_kt;
  const bool use_bias = a.n_slots > 0;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      uint32_t kv_iter = 0, item_iter = 0;
      uint32_t loads0 = 0, loads1 = 0;  // loads issued into stage 0 / 1
      bool ok = true;
      for (int64_t item = blockIdx.x; item < a.n_items && ok; item += gridDim.x, ++item_iter) {
        const int64_t qt = item % a.n_qt;
        const int64_t bh = item / a.n_qt;
        const int32_t h = static_cast<int32_t>(bh % H), b = static_cast<int32_t>(bh / H);
        if (item_iter > 0 && !mbar_wait(&bars->q_empty, (item_iter - 1) & 1, abort_flag, p.status,
                                        kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars->q_full, kQBytes);
        {
          const int32_t r = static_cast<int32_t>(qt * BM);
          tma_load_4d(q_s, &tm_q, &bars->q_full, 0, map_coord(a.oq, 1, r, h, b), map_coord(a.oq, 2, r, h, b),
                      map_coord(a.oq, 3, r, h, b));
        }
        for (int64_t j = 0; j < n_kt; ++j, ++kv_iter) {
          const uint32_t st = kv_iter % kStages, n = kv_iter / kStages;
          if (n > 0 && !mbar_wait(&bars->kv_empty[st], (n - 1) & 1, abort_flag, p.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          const bool bias_tile = use_bias && p.slot_tile_flags[qt * n_kt + j];
          mbar_arrive_expect_tx(&bars->kv_full[st], 2 * kKVBytes + (bias_tile ? kSlotBytes : 0));
          {
            const int32_t r = static_cast<int32_t>(j * BN);
            tma_load_4d(k_s + st * kKVBytes, &tm_k, &bars->kv_full[st], 0, map_coord(a.ok, 1, r, h, b),
                        map_coord(a.ok, 2, r, h, b), map_coord(a.ok, 3, r, h, b));
            tma_load_4d(v_s + st * kKVBytes, &tm_v, &bars->kv_full[st], 0, map_coord(a.ov, 1, r, h, b),
                        map_coord(a.ov, 2, r, h, b), map_coord(a.ov, 3, r, h, b));
          }
          if (bias_tile)
            bulk_load(slot_s + st * kSlotBytes, p.slots_packed + (qt * n_kt + j) * kSlotBytes, kSlotBytes,
                      &bars->kv_full[st]);
          if (st == 0) loads0 = n + 1; else loads1 = n + 1;
        }
      }
      // Drain: never leave a copy in flight into shared memory of an exiting CTA.
      if (item_iter > 0 || loads0 > 0) {
        volatile int32_t no_abort = 0;
        if (item_iter > 0) mbar_wait(&bars->q_full, (item_iter - 1) & 1, &no_abort, p.status, kDevTimeoutDrain);
        if (loads0 > 0) mbar_wait(&bars->kv_full[0], (loads0 - 1) & 1, &no_abort, p.status, kDevTimeoutDrain);
        if (loads1 > 0) mbar_wait(&bars->kv_full[1], (loads1 - 1) & 1, &no_abort, p.status, kDevTimeoutDrain);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const bool bf16 = p.dtype == 2;
      const uint32_t idesc_qk = idesc_f16(bf16, false, BM, BN);
      const uint32_t idesc_pv = idesc_f16(bf16, true, BM, HD);
      const uint32_t q_addr = smem_u32(q_s), k_addr = smem_u32(k_s), v_addr = smem_u32(v_s);
      uint32_t kv_iter = 0, s_iter = 0, pv_iter = 0, item_iter = 0;
      bool ok = true, issued = false;
      for (int64_t item = blockIdx.x; item < a.n_items && ok; item += gridDim.x, ++item_iter) {
        if (!mbar_wait(&bars->q_full, item_iter & 1, abort_flag, p.status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int64_t j = 0; j < n_kt && ok; ++j, ++kv_iter) {
          const uint32_t st = kv_iter % kStages;
          if (!mbar_wait(&bars->kv_full[st], (kv_iter / kStages) & 1, abort_flag, p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          const uint32_t sb = s_iter & 1, su = s_iter >> 1;
          if (su > 0 && !mbar_wait(&bars->s_free[sb], (su - 1) & 1, abort_flag, p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t s_col = tmem + (sb ? kColS1 : kColS0);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(q_addr + kk * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(k_addr + st * kKVBytes + kk * 32, 16, 1024);
            mma_ss(s_col, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          mma_commit(&bars->s_full[sb]);
          issued = true;
          ++s_iter;
          if (j > 0) {
            if (!mbar_wait(&bars->p_full, pv_iter & 1, abort_flag, p.status, kDevTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t pst = (kv_iter - 1) % kStages;
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
              const uint64_t bd = smem_desc_sw128(v_addr + pst * kKVBytes + kk * 2048, 8192, 1024);
              mma_ts(tmem + kColO, tmem + kColP + kk * 8, bd, idesc_pv, (j - 1 > 0 || kk > 0) ? 1u : 0u);
            }
            mma_commit(&bars->pv_done);
            mma_commit(&bars->kv_empty[pst]);
            ++pv_iter;
          }
        }
        if (!ok) break;
        mma_commit(&bars->q_empty);
        if (!mbar_wait(&bars->p_full, pv_iter & 1, abort_flag, p.status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t lst = (kv_iter - 1) % kStages;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bd = smem_desc_sw128(v_addr + lst * kKVBytes + kk * 2048, 8192, 1024);
          mma_ts(tmem + kColO, tmem + kColP + kk * 8, bd, idesc_pv, (n_kt - 1 > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bars->pv_done);
        mma_commit(&bars->kv_empty[lst]);
        ++pv_iter;
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
    const int32_t ns = a.n_slots;
    uint32_t s_iter = 0, kv_iter = 0, pv_iter = 0;
    bool ok = true;
    for (int64_t item = blockIdx.x; item < a.n_items && ok; item += gridDim.x) {
      const int64_t qt = item % a.n_qt;
      const int64_t bh = item / a.n_qt;
      const int64_t h = bh % H, b = bh / H;
      const int64_t i = qt * BM + row;  // token index of this thread's row
      if (use_bias) {
        // Per-query Look values, [slot][row] layout (bank = row % 32: conflict
        // free), pre-scaled to the log2 domain.  Only this thread reads its column.
        const bool valid = i >= 1 && i < N;
        const int64_t base = b * p.pose_stride[0] + (i - 1) * p.pose_stride[1] + h * p.pose_stride[2];
        if (a.pose_vec4) {
          const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.pose) + (valid ? base : 0));
          for (int s4 = 0; s4 < ns / 4; ++s4) {
            const float4 v4 = valid ? __ldg(src + s4) : make_float4(0.f, 0.f, 0.f, 0.f);
            table_s[(4 * s4 + 0) * BM + row] = v4.x * kLog2e;
            table_s[(4 * s4 + 1) * BM + row] = v4.y * kLog2e;
            table_s[(4 * s4 + 2) * BM + row] = v4.z * kLog2e;
            table_s[(4 * s4 + 3) * BM + row] = v4.w * kLog2e;
          }
        } else {
          for (int s = 0; s < ns; ++s)
            table_s[s * BM + row] =
                valid ? load_any(p.pose, base + s * p.pose_stride[3], p.pose_dtype) * kLog2e : 0.f;
        }
        table_s[ns * BM + row] = 0.f;
      }
      float m = -INFINITY, l = 0.f;
      uint64_t tile_mask = 0;  // bit k: key tile (j & ~63) + k carries Look bias
      for (int64_t j = 0; j < n_kt; ++j, ++kv_iter) {
        if (use_bias && (j & 63) == 0) {
          // Each warp gathers the flags of the next 64 key tiles with one ballot pair.
          const int64_t t0 = j + lane, t1 = j + 32 + lane;
          const bool f0 = t0 < n_kt && p.slot_tile_flags[qt * n_kt + t0] != 0;
          const bool f1 = t1 < n_kt && p.slot_tile_flags[qt * n_kt + t1] != 0;
          tile_mask = static_cast<uint64_t>(__ballot_sync(0xffffffffu, f0)) |
                      (static_cast<uint64_t>(__ballot_sync(0xffffffffu, f1)) << 32);
        }
        const uint32_t sb = s_iter & 1;
        if (!mbar_wait(&bars->s_full[sb], (s_iter >> 1) & 1, abort_flag, p.status, kDevTimeoutSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float2 t[BN / 2];  // t[c] holds keys 2c and 2c+1
        {
          uint32_t r0[16], r1[16], r2[16], r3[16];
          const uint32_t sa = lane_base + (sb ? kColS1 : kColS0);
          tmem_ld16(sa, r0);
          tmem_ld16(sa + 16, r1);
          tmem_ld16(sa + 32, r2);
          tmem_ld16(sa + 48, r3);
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
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->s_free[sb]);
        ++s_iter;

        // t holds raw scores on tiles without Look bias, and the log2-domain
        // logits scale*log2(e)*s + bias on tiles with it.
        const uint32_t st = kv_iter % kStages;
        const bool bias_tile = (tile_mask >> (j & 63)) & 1u;
        if (bias_tile) {
          if (!mbar_wait(&bars->kv_full[st], (kv_iter / kStages) & 1, abort_flag, p.status, kDevTimeoutSoftmax)) {
            ok = false;
            break;
          }
          const uint8_t* srow = slot_s + st * kSlotBytes + row * 16;
          const float* trow = table_s + row;
          const float2 c2 = make_float2(scale_log2, scale_log2);
#pragma unroll
          for (int c = 0; c < BN / 16; ++c) {
            const uint4 w = *reinterpret_cast<const uint4*>(srow + c * 2048);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const uint32_t s0 = __byte_perm(ww[e >> 2], 0u, 0x4440u | (e & 3));
              const uint32_t s1 = __byte_perm(ww[e >> 2], 0u, 0x4440u | ((e + 1) & 3));
              const float2 bias = make_float2(trow[s0 * BM], trow[s1 * BM]);
              t[c * 8 + e / 2] = fma2(t[c * 8 + e / 2], c2, bias);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->kv_empty[st]);

        if (j == n_kt - 1) {
          const int64_t key0 = j * BN;
#pragma unroll
          for (int c = 0; c < BN / 2; ++c) {
            if (key0 + 2 * c >= N) t[c].x = -INFINITY;
            if (key0 + 2 * c + 1 >= N) t[c].y = -INFINITY;
          }
        }
        float mx = row_max64(t);
        if (!bias_tile) mx *= scale_log2;

        bool waited_pv = false;
        if (j == 0) {
          m = mx;
        } else {
          const bool need = mx > m + kRescaleThreshold;
          if (__any_sync(0xffffffffu, need)) {
            if (!mbar_wait(&bars->pv_done, pv_iter & 1, abort_flag, p.status, kDevTimeoutSoftmax)) {
              ok = false;
              break;
            }
            waited_pv = true;
            tc_fence_after();
            const float f = need ? fast_exp2(m - mx) : 1.f;
            uint32_t r[16];
#pragma unroll
            for (int c = 0; c < HD / 16; ++c) {
              tmem_ld16(lane_base + kColO + c * 16, r);
              tmem_wait_ld();
              reg_fence16(r);
#pragma unroll
              for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * f);
              tmem_st16(lane_base + kColO + c * 16, r);
            }
            if (need) {
              l *= f;
              m = mx;
            }
          }
        }
        // exponents (log2 domain, relative to the running max), packed pairs
        const float2 nm2 = make_float2(-m, -m);
        const float2 c2 = bias_tile ? make_float2(1.f, 1.f) : make_float2(scale_log2, scale_log2);
        float2 part[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                          make_float2(0.f, 0.f)};
#pragma unroll
        for (int c = 0; c < BN / 2; ++c) {
          const float2 x = fma2(t[c], c2, nm2);
          t[c] = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          part[c & 3] = add2(part[c & 3], t[c]);
        }
        {
          const float2 s01 = add2(add2(part[0], part[1]), add2(part[2], part[3]));
          l += s01.x + s01.y;
        }
        // P region is free once the previous tile's PV MMA has completed.
        if (j > 0 && !waited_pv) {
          if (!mbar_wait(&bars->pv_done, pv_iter & 1, abort_flag, p.status, kDevTimeoutSoftmax)) {
            ok = false;
            break;
          }
        }
        if (j > 0) ++pv_iter;
        tc_fence_after();
        {
          uint32_t w0[16], w1[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            w0[e] = (p.dtype == 2) ? pack_bf16x2(t[e].x, t[e].y) : pack_f16x2(t[e].x, t[e].y);
            w1[e] = (p.dtype == 2) ? pack_bf16x2(t[16 + e].x, t[16 + e].y) : pack_f16x2(t[16 + e].x, t[16 + e].y);
          }
          tmem_st16(lane_base + kColP, w0);
          tmem_st16(lane_base + kColP + 16, w1);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full);
      }
      if (!ok) break;
      // Epilogue: wait for the item's last PV, normalise, store.
      if (!mbar_wait(&bars->pv_done, pv_iter & 1, abort_flag, p.status, kDevTimeoutSoftmax)) {
        ok = false;
        break;
      }
      ++pv_iter;
      tc_fence_after();
      const float inv = 1.f / l;
      uint32_t packed[HD / 2];
      {
        uint32_t r0[16], r1[16], r2[16], r3[16];
        tmem_ld16(lane_base + kColO, r0);
        tmem_ld16(lane_base + kColO + 16, r1);
        tmem_ld16(lane_base + kColO + 32, r2);
        tmem_ld16(lane_base + kColO + 48, r3);
        tmem_wait_ld();
        reg_fence16(r0);
        reg_fence16(r1);
        reg_fence16(r2);
        reg_fence16(r3);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          packed[e] = pack_out(r0[2 * e], r0[2 * e + 1], inv, p.dtype);
          packed[8 + e] = pack_out(r1[2 * e], r1[2 * e + 1], inv, p.dtype);
          packed[16 + e] = pack_out(r2[2 * e], r2[2 * e + 1], inv, p.dtype);
          packed[24 + e] = pack_out(r3[2 * e], r3[2 * e + 1], inv, p.dtype);
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
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// Builds a 4-D map (head_dim, then row / head / batch sorted by stride) over a
// (B, H, N, D) tensor with element strides `stride`, and reports where each
// logical coordinate lands.  Box: 64 x box_rows x 1 x 1 with 128-byte swizzle.
bool make_map(CUtensorMap* map, MapOrder* order, const void* base, const int64_t* stride, const SlaParams& p,
              uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const CUtensorMapDataType dt = p.dtype == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // logical outer dims: 0 = row (seq), 1 = head, 2 = batch
  const int64_t ext[3] = {p.seq, p.heads, p.batch};
  const int64_t str[3] = {stride[2], stride[1], stride[0]};
  const uint32_t bx[3] = {box_rows, 1, 1};
  int idx[3] = {0, 1, 2};
  for (int x = 0; x < 3; ++x)
    for (int y = x + 1; y < 3; ++y)
      if (str[idx[y]] < str[idx[x]] || (str[idx[y]] == str[idx[x]] && idx[y] < idx[x])) {
        const int tmp = idx[x];
        idx[x] = idx[y];
        idx[y] = tmp;
      }
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(p.head_dim), 0, 0, 0};
  cuuint64_t strides[3];
  cuuint32_t box[4] = {static_cast<cuuint32_t>(HD), 1, 1, 1};
  int8_t pos[3];
  for (int x = 0; x < 3; ++x) {
    dims[x + 1] = static_cast<cuuint64_t>(ext[idx[x]]);
    strides[x] = static_cast<cuuint64_t>(str[idx[x]]) * 2;
    box[x + 1] = bx[idx[x]];
    pos[idx[x]] = static_cast<int8_t>(x + 1);
  }
  order->row = pos[0];
  order->head = pos[1];
  order->batch = pos[2];
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tma_stride_ok(const void* base, const int64_t* stride) {
  if (reinterpret_cast<uintptr_t>(base) % 16) return false;
  if (stride[3] != 1) return false;
  for (int d = 0; d < 3; ++d) {
    if (stride[d] <= 0) return false;
    if ((stride[d] * 2) % 16) return false;
    if (stride[d] * 2 >= (int64_t(1) << 40)) return false;
  }
  return true;
}

uint32_t table_bytes_for(int32_t n_slots) {
  return n_slots > 0 ? static_cast<uint32_t>((n_slots + 1) * BM * sizeof(float)) : 0u;
}

size_t smem_bytes_for(uint32_t table_bytes) {
  size_t bytes = 1024 + SmemLayout::table + table_bytes + sizeof(Barriers) + 64;
  // Keep at most two CTAs per SM so two TMEM allocations of 256 columns fit.
  const size_t floor_bytes = 80 * 1024;
  return bytes < floor_bytes ? floor_bytes : bytes;
}

}  // namespace

int32_t sla_tc_supported(const SlaParams& p) {
  if (p.dtype != 1 && p.dtype != 2) return 0;
  if (p.head_dim != HD) return 0;
  if (p.dense != nullptr) return 0;
  if (p.bias_mode != 0 && p.bias_mode != 2) return 0;
  if (p.bias_mode == 2 && (p.poses < 1 || p.poses > kMaxSlots || !p.slots_packed || !p.slot_tile_flags)) return 0;
  if (p.status == nullptr) return 0;
  if (p.seq < 2 || p.seq > (int64_t(1) << 30) || p.batch > (int64_t(1) << 30) || p.heads > (int64_t(1) << 30))
    return 0;
  if (!(p.scale > 0.f) || !(p.scale < 3.0e38f)) return 0;
  if (!tma_stride_ok(p.q, p.q_stride) || !tma_stride_ok(p.k, p.k_stride) || !tma_stride_ok(p.v, p.v_stride))
    return 0;
  if (reinterpret_cast<uintptr_t>(p.out) % 16 || p.out_stride[3] != 1) return 0;
  for (int d = 0; d < 3; ++d)
    if ((p.out_stride[d] * 2) % 16) return 0;
  if (!get_encode_fn()) return 0;
  return 1;
}

int32_t launch_sla_tc(const SlaParams& p, cudaStream_t stream, int sm_count) {
  if (!sla_tc_supported(p)) return 8;
  CUtensorMap mq, mk, mv;
  TcArgs a;
  if (!make_map(&mq, &a.oq, p.q, p.q_stride, p, BM) || !make_map(&mk, &a.ok, p.k, p.k_stride, p, BN) ||
      !make_map(&mv, &a.ov, p.v, p.v_stride, p, BN))
    return 4;
  a.p = p;
  a.n_qt = (p.seq + BM - 1) / BM;
  a.n_kt = (p.seq + BN - 1) / BN;
  a.n_items = p.batch * p.heads * a.n_qt;
  a.n_slots = p.bias_mode == 2 ? static_cast<int32_t>(p.poses) : 0;
  a.table_bytes = table_bytes_for(a.n_slots);
  a.pose_vec4 = 0;
  if (a.n_slots > 0 && p.pose_dtype == 0 && p.pose_stride[3] == 1 && a.n_slots % 4 == 0 &&
      reinterpret_cast<uintptr_t>(p.pose) % 16 == 0 && p.pose_stride[0] % 4 == 0 && p.pose_stride[1] % 4 == 0 &&
      p.pose_stride[2] % 4 == 0)
    a.pose_vec4 = 1;
  const size_t smem = smem_bytes_for(a.table_bytes);
  if (cudaFuncSetAttribute(sla_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
          cudaSuccess ||
      cudaFuncSetAttribute(sla_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return 6;
  // Resident CTAs per SM from the register and shared-memory budgets (the
  // occupancy query does not account for the carveout set above).
  int dev = 0, smem_per_sm = 0, regs_per_sm = 0;
  cudaFuncAttributes fa;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaFuncGetAttributes(&fa, sla_tc_kernel) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&regs_per_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev) != cudaSuccess)
    return 6;
  const int warp_regs = ((fa.numRegs * 32 + 255) / 256) * 256;
  const int by_regs = regs_per_sm / (warp_regs * (kThreads / 32));
  const int by_smem = smem_per_sm / static_cast<int>(smem + 1024);
  int per_sm = by_regs < by_smem ? by_regs : by_smem;
  if (per_sm > 2) per_sm = 2;  // two 256-column TMEM allocations per SM
  if (per_sm < 1) return 6;
  int64_t grid = static_cast<int64_t>(sm_count) * per_sm;
  if (grid > a.n_items) grid = a.n_items;
  sla_tc_kernel<<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(mq, mk, mv, a);
  return cudaGetLastError() == cudaSuccess ? 0 : 6;
}

}  // namespace intp
