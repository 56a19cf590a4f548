// sla_internal.h - kernel-side parameter block shared by the Look-attention
// kernels and the C-ABI dispatcher (capi.cu).  Not part of the public ABI.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace intp {

struct SlaParams {
  int64_t batch, heads, seq, head_dim;
  float scale;
  int32_t dtype;
  const void* q; int64_t q_stride[4];
  const void* k; int64_t k_stride[4];
  const void* v; int64_t v_stride[4];
  void* out; int64_t out_stride[4];
  float* lse;
  int32_t bias_mode;  // 0 none, 1 fields, 2 slots, 3 slot fields
  int64_t poses;      // P (modes 1, 3) or number of slots (mode 2)
  int64_t slots;      // number of slots (mode 3)
  const void* pose; int64_t pose_stride[4]; int32_t pose_dtype;
  const void* fields; int64_t fields_stride[4]; int32_t fields_dtype;
  const uint8_t* slots_packed;
  const uint8_t* slot_tile_flags;
  const void* dense; int64_t dense_stride[4]; int32_t dense_dtype;
  int32_t* status;
};

// Packed slot-table geometry (shared by the host packer and both kernels):
// tiles of 128 query tokens x 64 key tokens, 8192 bytes each, stored
// [q_tile][k_tile][key_chunk(4)][query(128)][16 keys].  Entry = slot index,
// or n_slots for "no Look bias" (CLS row/column, padding, unslotted pairs).
constexpr int kSlotTileQ = 128;
constexpr int kSlotTileK = 64;
constexpr int kSlotTileBytes = kSlotTileQ * kSlotTileK;

// Backward pass parameters: the forward's (q, k, v, out = forward output,
// lse = forward LSE, bias inputs) plus the output gradient and fp32 result
// buffers (each may be null when not wanted).
struct SlaBwdParams {
  SlaParams f;
  const void* grad_out; int64_t grad_out_stride[4];
  float* grad_q; float* grad_k; float* grad_v;  // (B,H,N,D) contiguous
  float* grad_pose;                              // (B,Np,H,P) contiguous
  float* grad_fields;                            // (H,P,Np,Np) contiguous, zero-filled (FIELDS mode)
  float* grad_dense;                             // (B,H,Np,Np) contiguous
  float* delta;                                  // (B,H,N) scratch
};

int32_t launch_sla_simt(const SlaParams& p, cudaStream_t stream);
int32_t launch_sla_backward(const SlaBwdParams& bp, cudaStream_t stream);
int32_t launch_nl1_backward(const float* x, const float* w, const float* grad_out, float* grad_x, float* grad_w,
                            int64_t rows, int64_t protos, int64_t features, cudaStream_t stream);
// Returns INTP_ERR_UNSUPPORTED (8) when the tensor-core path does not apply.
int32_t launch_sla_tc(const SlaParams& p, cudaStream_t stream, int sm_count);
// 1 when one of the two tensor-core kernels takes the request.
int32_t sla_tc_supported(const SlaParams& p);
// Requirements both tensor-core kernels share (look_attention_tc.cu).
int32_t tc_common_ok(const SlaParams& p);
// The tiled tensor-core kernel (any N; no dense bias, no general fields).
int32_t sla_long_supported(const SlaParams& p);
// The single-pass tensor-core kernel for sequences of at most 256 tokens
// (look_attention_short.cu, every bias mode and dense bias); launch_sla_tc
// prefers it when it applies.
int32_t sla_short_supported(const SlaParams& p);
int32_t launch_sla_short(const SlaParams& p, cudaStream_t stream, int sm_count);
// Tensor-core probability / score-gradient pass (backward_tc.cu); returns
// INTP_ERR_UNSUPPORTED (8) when the inputs do not qualify.
int32_t launch_sla_probability_score_grad(const SlaParams& p, const void* dout, const int64_t* dout_stride,
                                          void* probability, void* score_grad, int64_t ld, float* grad_pose,
                                          cudaStream_t stream);
// Fused tensor-core backward (backward_fused.cu): dQ / delta / slot gradient,
// then dK / dV.  `slots_t` is the transposed packed slot table (SLOTS mode).
int32_t sla_backward_fused_supported(const SlaBwdParams& bp, const uint8_t* slots_t);
int32_t launch_sla_backward_fused(const SlaBwdParams& bp, const uint8_t* slots_t, cudaStream_t stream);
int32_t launch_nl1(const float* x, const float* w, float* out, int64_t rows, int64_t protos, int64_t features,
                   cudaStream_t stream);

}  // namespace intp
