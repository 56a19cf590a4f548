// sla_look_table.cuh - the per-query Look table of the tensor-core kernels.
//
// Both tensor-core Look-attention kernels turn the Look bias of a 128-query
// tile into a shared-memory table laid out [slot][row] (row = query within the
// tile, one fp32 column per row: a warp reading one slot per lane touches 32
// different banks), pre-scaled to the log2 domain, with two extra entries per
// row: "no bias" (0) and "key past the sequence end" (-inf).  The score tiles
// then gather from it through the packed pair table.
//
//   SLOTS       : table[s][row] = log2(e) * pose[b, i-1, h, s]
//   SLOT_FIELDS : table[s][row] = log2(e) * sum_p pose[b, i-1, h, p] * slot_fields[h, p, s]
//                 (model/deit_tiny_rot_hex_look.py:397-451 feeds exactly this
//                 product to the attention as pose x fields)
//
// The functions are templates over the kernel's argument block `A`, which
// provides: p (SlaParams), n_slots, n_poses, pose_vec4 (pose rows are 16-byte
// aligned fp32 with unit stride along slots / poses) and sf_vec4 (slot_fields
// rows likewise: they are then staged in shared memory by stage_slot_fields).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "sla_internal.h"
#include "sm100_ptx.cuh"

namespace intp {

constexpr int kTableRows = 128;             // queries per tile (one table column each)
constexpr float kLog2eF = 1.4426950408889634f;
constexpr int kMaxLookSlots = 93;           // slots the tensor-core kernels take
constexpr int kMaxLookPoses = 16;           // SLOT_FIELDS: Look poses per head
constexpr int kModelLookPoses = 12;         // the half6d3r Look bank: 2 supports x 6 directions

__device__ __forceinline__ float load_any(const void* p, int64_t idx, int32_t dtype) {
  switch (dtype) {
    case 1: return __half2float(static_cast<const __half*>(p)[idx]);
    case 2: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
    default: return static_cast<const float*>(p)[idx];
  }
}

// SLOTS: query token i's Look values into column `row` of the table (only this
// thread reads its column).  Rows past the sequence and the CLS token get 0.
template <class A>
__device__ __forceinline__ void stage_table(float* table_s, const A& a, int64_t b, int64_t h, int64_t i, int row) {
  constexpr int BM = kTableRows;
  const SlaParams& p = a.p;
  const int32_t ns = a.n_slots;
  const bool valid = i >= 1 && i < p.seq;
  const int64_t base = b * p.pose_stride[0] + (i - 1) * p.pose_stride[1] + h * p.pose_stride[2];
  if (a.pose_vec4) {
    // The whole row's 16-byte loads in flight at once: one memory round trip
    // (an L2 hit when the previous item prefetched it).
    constexpr int kMaxVec = kMaxLookSlots / 4;
    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.pose) + (valid ? base : 0));
    float4 v4[kMaxVec];
#pragma unroll
    for (int u = 0; u < kMaxVec; ++u)
      v4[u] = (valid && u < ns / 4) ? __ldg(src + u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < kMaxVec; ++u) {
      if (u < ns / 4) {
        float* dst = table_s + 4 * u * BM + row;
        dst[0] = v4[u].x * kLog2eF;
        dst[BM] = v4[u].y * kLog2eF;
        dst[2 * BM] = v4[u].z * kLog2eF;
        dst[3 * BM] = v4[u].w * kLog2eF;
      }
    }
  } else {
    for (int s = 0; s < ns; ++s)
      table_s[s * BM + row] = valid ? load_any(p.pose, base + s * p.pose_stride[3], p.pose_dtype) * kLog2eF : 0.f;
  }
  table_s[ns * BM + row] = 0.f;               // "no bias"
  table_s[(ns + 1) * BM + row] = -INFINITY;   // key past the sequence end
}

// SLOT_FIELDS with sf_vec4: threads tid = 0, stride, 2 stride, ... copy head h's
// slot values (P rows of S fp32) into `sf` (shared memory).
template <class A>
__device__ __forceinline__ void stage_slot_fields(float* sf, const A& a, int64_t h, int tid, int stride) {
  const SlaParams& p = a.p;
  const int groups = a.n_slots / 4, total = a.n_poses * groups;
  const float* src = static_cast<const float*>(p.fields) + h * p.fields_stride[0];
  float4* dst = reinterpret_cast<float4*>(sf);
  for (int idx = tid; idx < total; idx += stride) {
    const int pp = idx / groups, s4 = idx - pp * groups;
    dst[idx] = __ldg(reinterpret_cast<const float4*>(src + pp * p.fields_stride[1]) + s4);
  }
}

// SLOT_FIELDS: query token i's Look pose row (raw values; rows past the
// sequence and the CLS token read as 0).
template <class A>
__device__ __forceinline__ void load_pose_row(float (&w)[kMaxLookPoses], const A& a, int64_t b, int64_t h, int64_t i) {
  const SlaParams& p = a.p;
  const int32_t np = a.n_poses;
  const bool valid = i >= 1 && i < p.seq;
  const int64_t base = b * p.pose_stride[0] + (i - 1) * p.pose_stride[1] + h * p.pose_stride[2];
  if (a.pose_vec4) {
    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.pose) + (valid ? base : 0));
#pragma unroll
    for (int c = 0; c < kMaxLookPoses / 4; ++c) {
      const float4 v = (valid && 4 * c < np) ? __ldg(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      w[4 * c] = v.x;
      w[4 * c + 1] = v.y;
      w[4 * c + 2] = v.z;
      w[4 * c + 3] = v.w;
    }
  } else if (p.pose_dtype == 0) {
    const float* src = static_cast<const float*>(p.pose);
#pragma unroll
    for (int pp = 0; pp < kMaxLookPoses; ++pp)
      w[pp] = (valid && pp < np) ? __ldg(src + base + pp * p.pose_stride[3]) : 0.f;
  } else {
#pragma unroll
    for (int pp = 0; pp < kMaxLookPoses; ++pp)
      w[pp] = (valid && pp < np) ? load_any(p.pose, base + pp * p.pose_stride[3], p.pose_dtype) : 0.f;
  }
}

// Table columns of one warp in SLOT_FIELDS mode.  Lane (gp = lane / 8,
// rb = lane % 8) takes rows rb + 8 ((gp + m) % 4), m = 0..3 (their poses by
// shuffle from the owning lanes) and the 4-slot groups gp, gp + 4, ...: each
// 16-byte slot-value load feeds four rows (16 independent FMA chains), and for a
// fixed m the 32 lanes store to 32 different rows (banks).  P, the number of
// poses, is a compile-time constant (no per-pose tests).
template <int P>
__device__ __forceinline__ void build_rows_sf(float* col0, const float4* sf, int groups, int gp, int rb,
                                              const float (&w)[kMaxLookPoses]) {
  constexpr int BM = kTableRows;
  int rows[4];
  float wr[4][P];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    rows[m] = rb + 8 * ((gp + m) & 3);
#pragma unroll
    for (int pp = 0; pp < P; ++pp) wr[m][pp] = __shfl_sync(0xffffffffu, w[pp], rows[m]);
  }
  for (int g = gp; g < groups; g += 4) {
    float2 acc[4][2];  // packed fp32 pairs: slots (4g, 4g+1) and (4g+2, 4g+3) of row m
#pragma unroll
    for (int m = 0; m < 4; ++m) acc[m][0] = acc[m][1] = make_float2(0.f, 0.f);
#pragma unroll
    for (int pp = 0; pp < P; ++pp) {
      const float4 f = sf[pp * groups + g];
      const float2 f01 = make_float2(f.x, f.y), f23 = make_float2(f.z, f.w);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float2 w2 = make_float2(wr[m][pp], wr[m][pp]);
        acc[m][0] = fma2(w2, f01, acc[m][0]);
        acc[m][1] = fma2(w2, f23, acc[m][1]);
      }
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      float* dst = col0 + 4 * g * BM + rows[m];
      dst[0] = acc[m][0].x;
      dst[BM] = acc[m][0].y;
      dst[2 * BM] = acc[m][1].x;
      dst[3 * BM] = acc[m][1].y;
    }
  }
}

// SLOT_FIELDS: the table built from the query's Look pose (w, this thread's
// row; scaled in place to the log2 domain) and the head's slot fields.  With
// sf_vec4 the slot values come from `sf` (staged in shared memory) and each
// lane computes four rows of its warp; otherwise each thread computes its own
// row from global memory.  Every lane of the warp must call this together.
template <class A>
__device__ __forceinline__ void build_table_sf(float* table_s, const float* sf_s, const A& a, int64_t h, int row,
                                               float (&w)[kMaxLookPoses]) {
  constexpr int BM = kTableRows;
  const SlaParams& p = a.p;
  const int32_t ns = a.n_slots, np = a.n_poses;
#pragma unroll
  for (int pp = 0; pp < kMaxLookPoses; ++pp) w[pp] *= kLog2eF;
  if (a.sf_vec4) {
    const float4* sf = reinterpret_cast<const float4*>(sf_s);
    const int groups = ns / 4;
    const int lane = row & 31, gp = lane >> 3, rb = lane & 7;
    float* col0 = table_s + (row - lane);  // column of the warp's first row
    if (np == kModelLookPoses) {
      build_rows_sf<kModelLookPoses>(col0, sf, groups, gp, rb, w);
    } else {
      // other pose counts: each thread its own row, one 4-slot group at a time
      for (int g = 0; g < groups; ++g) {
        float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
#pragma unroll
        for (int pp = 0; pp < kMaxLookPoses; ++pp) {
          if (pp < np) {
            const float4 f = sf[pp * groups + g];
            lo = fma2(make_float2(w[pp], w[pp]), make_float2(f.x, f.y), lo);
            hi = fma2(make_float2(w[pp], w[pp]), make_float2(f.z, f.w), hi);
          }
        }
        float* dst = col0 + 4 * g * BM + lane;
        dst[0] = lo.x;
        dst[BM] = lo.y;
        dst[2 * BM] = hi.x;
        dst[3 * BM] = hi.y;
      }
    }
    __syncwarp();
  } else {
    for (int s = 0; s < ns; ++s) {
      float acc = 0.f;
#pragma unroll
      for (int pp = 0; pp < kMaxLookPoses; ++pp)
        if (pp < np)
          acc = fmaf(w[pp],
                     load_any(p.fields, h * p.fields_stride[0] + pp * p.fields_stride[1] + s * p.fields_stride[2],
                              p.fields_dtype),
                     acc);
      table_s[s * BM + row] = acc;
    }
  }
  table_s[ns * BM + row] = 0.f;               // "no bias"
  table_s[(ns + 1) * BM + row] = -INFINITY;   // key past the sequence end
}

// Starts fetching into L2 the Look row that stage_table will read for query
// token i of (b, h) in a later work item.
template <class A>
__device__ __forceinline__ void prefetch_table_row(const A& a, int64_t b, int64_t h, int64_t i) {
  const SlaParams& p = a.p;
  if (!a.pose_vec4 || i < 1 || i >= p.seq) return;
  const int64_t base = b * p.pose_stride[0] + (i - 1) * p.pose_stride[1] + h * p.pose_stride[2];
  bulk_prefetch_l2(static_cast<const float*>(p.pose) + base, static_cast<uint32_t>(a.n_slots) * 4u);
}

}  // namespace intp
