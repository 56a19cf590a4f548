// sla_tc_common.cuh - pieces shared by the two tensor-core Look-attention
// kernels (look_attention_tc.cu for any sequence length, look_attention_short.cu
// for sequences of at most 256 tokens): TMA tensor maps over (B, H, N, D)
// tensors with arbitrary strides, and the layout checks they need.
#pragma once
#include <cuda.h>
#include <cstdint>
#include "sla_internal.h"
#include "tma_host.h"

namespace intp {

// Position (1..3) of the row / head / batch coordinate in a tensor map whose
// outer dimensions are sorted by increasing stride (dimension 0 is head_dim).
struct MapOrder {
  int8_t row, head, batch;
};

// TMA coordinates {0, c1, c2, c3} with row / head / batch placed per `o`.
__device__ __forceinline__ int32_t map_coord(const MapOrder& o, int pos, int32_t row, int32_t head, int32_t batch) {
  return o.row == pos ? row : (o.head == pos ? head : batch);
}

inline EncodeTiledFn get_encode_fn() { return tensor_map_encoder(); }

// Builds a 4-D map (head_dim, then row / head / batch sorted by stride) over a
// (B, H, N, D) tensor with element strides `stride`, and reports where each
// logical coordinate lands.  Box: 64 x box_rows x 1 x 1 with 128-byte swizzle
// (box_rows <= 256).  Rows past N read as zero.
inline bool make_map(CUtensorMap* map, MapOrder* order, const void* base, const int64_t* stride, const SlaParams& p,
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
  cuuint32_t box[4] = {64u, 1, 1, 1};
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

// A (B, H, N, 64) 16-bit tensor TMA can read: 16-byte aligned base, unit
// head_dim stride, other strides positive multiples of 16 bytes.
inline bool tma_stride_ok(const void* base, const int64_t* stride) {
  if (reinterpret_cast<uintptr_t>(base) % 16) return false;
  if (stride[3] != 1) return false;
  for (int d = 0; d < 3; ++d) {
    if (stride[d] <= 0) return false;
    if ((stride[d] * 2) % 16) return false;
    if (stride[d] * 2 >= (int64_t(1) << 40)) return false;
  }
  return true;
}

// Budget of the pipeline waits of the tensor-core kernels (nanoseconds); set by
// intp_set_wait_budget_ns, one second by default.
uint64_t tc_wait_budget_ns();

}  // namespace intp
