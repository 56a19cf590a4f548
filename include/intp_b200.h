/*
 * intp_b200.h - C ABI of the B200 (sm_100a) Look-attention and negative-L1 library.
 *
 * The reference (Hevensh/INTP_Preliminary) is pure Python + Triton, so it has no
 * native FFI of its own.  Each entry point below replaces one Python-level
 * launch site of the reference and takes exactly the arguments that site hands
 * to its Triton kernel: raw device pointers, element strides, sizes, a dtype
 * code and the CUDA stream.  No torch type crosses this boundary, no C++
 * exception escapes it, and the library never allocates or frees caller memory.
 *
 * Every function returns an intp_status (0 = success).
 */
#ifndef INTP_B200_H
#define INTP_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define INTP_API __attribute__((visibility("default")))
#else
#define INTP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
typedef int32_t intp_status;
#define INTP_OK               0
#define INTP_ERR_ARGUMENT     1  /* null pointer or inconsistent sizes          */
#define INTP_ERR_SHAPE        2  /* shape rule of the reference violated        */
#define INTP_ERR_DTYPE        3  /* unsupported dtype code                      */
#define INTP_ERR_LAYOUT       4  /* stride / alignment the kernel cannot take   */
#define INTP_ERR_ARCH         5  /* device is not sm_100 (B200)                 */
#define INTP_ERR_LAUNCH       6  /* CUDA runtime error at launch                */
#define INTP_ERR_TIMEOUT      7  /* a bounded device wait gave up (see status)  */
#define INTP_ERR_UNSUPPORTED  8  /* valid request outside the kernel's coverage */

/* ---- dtype codes --------------------------------------------------------- */
#define INTP_F32   0
#define INTP_F16   1
#define INTP_BF16  2

/* ---- Look-bias modes ------------------------------------------------------ */
/* NONE    : plain softmax attention (no Look bias).
 * FIELDS  : the reference's general form: bias[b,h,i,j] =
 *           sum_p pose[b,i-1,h,p] * fields[h,p,i-1,j-1] for i,j >= 1.
 * SLOTS   : the same bias when fields[h,p,q,k] is the one-hot indicator of a
 *           per-pair slot index: bias[b,h,i,j] = pose[b,i-1,h,slot(i,j)]
 *           (zero where the pair has no slot).  The pair table is prepared
 *           once by sla_pack_slot_table and shared by every batch and head.
 * SLOT_FIELDS : FIELDS when each field is a per-slot value gathered by the same
 *           pair table: fields[h,p,i-1,j-1] = slot_fields[h,p,slot(i,j)], so
 *           bias[b,h,i,j] = sum_p pose[b,i-1,h,p] * slot_fields[h,p,slot(i,j)]
 *           (zero where the pair has no slot).  This is the reference model's
 *           Look-bank call (model/deit_tiny_rot_hex_look.py:397-451 ->
 *           layers/mini_vit.py:103) with its (H, P, Np, Np) fields held as
 *           (H, P, S) slot values: `fields` = slot_fields, `poses` = P,
 *           `slots` = S.                                                    */
#define SLA_BIAS_NONE         0
#define SLA_BIAS_FIELDS       1
#define SLA_BIAS_SLOTS        2
#define SLA_BIAS_SLOT_FIELDS  3

/* Slot value meaning "no Look bias for this pair" in an unpacked slot table. */
#define SLA_SLOT_NONE 255

/* Kernel selection (sla_forward_args.kernel). */
#define SLA_KERNEL_AUTO      0   /* tcgen05 path when it applies, else SIMT     */
#define SLA_KERNEL_SIMT      1   /* CUDA-core path (every dtype, mode, layout)  */
#define SLA_KERNEL_TCGEN05   2   /* tensor-core path; fails if it cannot apply  */

/* Arguments of one structured-Look-attention forward.
 *
 * Tensors follow the reference layouts (layers/triton_structured_look_attention.py:412-424):
 *   q, k, v, out : (B, H, N, D), N = Np + 1 (token 0 is CLS), any strides, D stride 1
 *   pose         : (B, Np, H, P) floating, any strides
 *   fields       : (H, P, Np, Np) floating (FIELDS mode), any strides;
 *                  (H, P, S) slot_fields (SLOT_FIELDS mode), strides [0..2]
 *   dense        : (B, H, Np, Np) floating or NULL, any strides
 *   lse          : (B, H, N) float32 contiguous, or NULL when not wanted
 * Strides are in elements.  In SLOTS and SLOT_FIELDS modes `slots_packed` /
 * `slot_tile_flags` come from sla_pack_slot_table for this N and are device
 * pointers.                                                                 */
typedef struct sla_forward_args {
  int64_t batch, heads, seq, head_dim;
  float scale;
  int32_t dtype;                 /* dtype of q, k, v and out                  */
  const void* q; int64_t q_stride[4];
  const void* k; int64_t k_stride[4];
  const void* v; int64_t v_stride[4];
  void* out;     int64_t out_stride[4];
  float* lse;
  int32_t bias_mode;
  int64_t poses;                 /* P (FIELDS, SLOT_FIELDS) or slots (SLOTS)  */
  const void* pose;   int64_t pose_stride[4];   int32_t pose_dtype;
  const void* fields; int64_t fields_stride[4]; int32_t fields_dtype;
  const uint8_t* slots_packed;
  const uint8_t* slot_tile_flags;
  const void* dense;  int64_t dense_stride[4];  int32_t dense_dtype;
  int32_t* status;               /* device int32: bounded-wait error word     */
  int32_t kernel;                /* SLA_KERNEL_*                              */
  int64_t slots;                 /* S, number of slots (SLOT_FIELDS mode)     */
} sla_forward_args;

/* Structured Look attention forward.
 * Replaces the launch of `_structured_look_forward` in
 * `_StructuredLookAttention.forward` (layers/triton_structured_look_attention.py:297-338),
 * reached through `structured_look_attention` (:412-424).  `stream` is a
 * cudaStream_t.  The call is asynchronous; device-side wait failures are
 * reported through *args->status (read it with sla_read_status).            */
INTP_API intp_status sla_forward(const sla_forward_args* args, void* stream);

/* Arguments of the structured-Look-attention backward.  `fwd` repeats the
 * forward call (fwd.out = the forward output O, fwd.lse = its LSE, required),
 * grad_out is dL/dO with the layout rules of q.  Results are float32,
 * contiguous, and each may be NULL when not wanted:
 *   grad_q, grad_k, grad_v : (B, H, N, D)
 *   grad_pose              : (B, Np, H, P)   (FIELDS and SLOTS modes; in SLOTS
 *                            mode P = number of slots: dL/d per-slot value)
 *   grad_fields            : (H, P, Np, Np)  (FIELDS mode; zero-filled by the
 *                            caller, accumulated with atomics over the batch)
 *   grad_dense             : (B, H, Np, Np)  (when fwd.dense is set)
 * delta: (B, H, N) float32 scratch (receives rowsum(dO * O)).
 * slots_packed_t: SLOTS mode, the tensor-core path only: the slot table
 * transposed (slots_t[k][q] = slots[q][k]) and packed by sla_pack_slot_table
 * (same sizes as fwd.slots_packed); NULL keeps SLOTS on the CUDA-core path.  */
typedef struct sla_backward_args {
  sla_forward_args fwd;
  const void* grad_out; int64_t grad_out_stride[4];
  float* grad_q; float* grad_k; float* grad_v;
  float* grad_pose;
  float* grad_fields;
  float* grad_dense;
  float* delta;
  const uint8_t* slots_packed_t;
} sla_backward_args;

/* Structured Look attention backward.  Replaces the launch of
 * `_structured_look_probability_score_grad` and the batched matmuls that follow
 * it in `_StructuredLookAttention.backward`
 * (layers/triton_structured_look_attention.py:172-292, 341-409); flash-style:
 * P is recomputed from the LSE, no N x N buffer is needed beyond grad_dense.
 * fwd.kernel selects the implementation: SLA_KERNEL_AUTO takes the tensor
 * cores (two tcgen05 kernels: dQ with delta and the slot gradient per query
 * tile, then dK and dV per key tile; bf16 / f16, head_dim 64, no bias or SLOTS
 * with slots_packed_t, no dense bias, no grad_fields) when the request
 * qualifies and the CUDA cores otherwise; SLA_KERNEL_SIMT forces the CUDA
 * cores; SLA_KERNEL_TCGEN05 returns INTP_ERR_UNSUPPORTED when the tensor-core
 * path cannot take the request.  Deterministic on both paths except FIELDS
 * grad_fields (atomics over the batch).                                      */
INTP_API intp_status sla_backward(const sla_backward_args* args, void* stream);

/* Probability / score-gradient pass of the backward on the tensor cores: the
 * direct replacement of `_structured_look_probability_score_grad`
 * (layers/triton_structured_look_attention.py:172-292, launched at :350-368).
 * Writes, for every (b, h, query, key < N),
 *   probability[b,h,q,k] = exp(scale q.k + bias - lse)
 *   score_grad[b,h,q,k]  = probability * (dO.v_k - rowsum(dO * O))
 * in fwd.dtype, row-major (B, H, N, ld); columns N .. round_up(N, 8) - 1 of
 * each row receive 0, columns from round_up(N, 8) on are left untouched.
 * The caller finishes the backward with the reference's batched products
 * (:371-376): dQ = scale score_grad K, dK = scale score_grad^T Q,
 * dV = probability^T dO.  With SLOTS bias, grad_pose (B, N-1, H, n_slots)
 * fp32 (may be NULL) receives the per-slot sums of score_grad of each query
 * row, which is the reference's grad_pose through one-hot fields (:378-395).
 * Takes bf16 / f16, head_dim 64, bias NONE or SLOTS, no dense bias; anything
 * else returns INTP_ERR_UNSUPPORTED (sla_backward covers it).  Needs fwd.lse;
 * ld >= N, ld % 8 == 0, both outputs 16-byte aligned (INTP_ERR_LAYOUT).
 * Errors inside the kernel (a wait that ran out) land in fwd.status.        */
typedef struct sla_probability_score_grad_args {
  sla_forward_args fwd;
  const void* grad_out; int64_t grad_out_stride[4];
  void* probability;
  void* score_grad;
  int64_t ld;
  float* grad_pose;
} sla_probability_score_grad_args;

INTP_API intp_status sla_probability_score_grad(const sla_probability_score_grad_args* args, void* stream);

/* Bytes needed by the packed slot table and the tile flags for sequence N. */
INTP_API intp_status sla_slot_table_bytes(int64_t seq, int64_t* packed_bytes, int64_t* flag_bytes);

/* Host-side packing of a (Np x Np) uint8 slot table (SLA_SLOT_NONE = no bias,
 * other values < n_slots <= 253) into the tile layout the kernels read
 * (tiles of 128 query x 64 key tokens; entry n_slots = no bias, n_slots + 1 =
 * key past the sequence end, which the kernels treat as masked).  Pure CPU:
 * both outputs are host buffers of the sizes sla_slot_table_bytes returns.
 * Stands in for the one-hot `fields` tensor of the reference API
 * (layers/triton_structured_look_attention.py:116-130 loads it per pair).   */
INTP_API intp_status sla_pack_slot_table(const uint8_t* slots, int64_t patch_count, int32_t n_slots,
                                uint8_t* packed, uint8_t* tile_flags);

/* Negative L1 distance: out[m,p] = -sum_f |x[m,f] - w[p,f]|, float32, all
 * row-major contiguous.  Replaces the launch of `_negative_l1_forward` in
 * `_TritonNegativeL1.forward` (layers/triton_negative_l1.py:157-187), reached
 * through `negative_l1_distance` (:233-241).                                  */
INTP_API intp_status nl1_forward(const float* x, const float* w, float* out,
                        int64_t rows, int64_t protos, int64_t features, void* stream);

/* Negative-L1 backward (float32, row-major contiguous; sign(0) = 0):
 *   grad_x[m,f] = -sum_p grad_out[m,p] * sign(x[m,f] - w[p,f])
 *   grad_w[p,f] =  sum_m grad_out[m,p] * sign(x[m,f] - w[p,f])
 * Either output may be NULL.  Replaces `_negative_l1_backward_x/_w`
 * (layers/triton_negative_l1.py:55-154, launched at :189-230).              */
INTP_API intp_status nl1_backward(const float* x, const float* w, const float* grad_out, float* grad_x,
                         float* grad_w, int64_t rows, int64_t protos, int64_t features, void* stream);

/* Dense Look-grid sampling: out[b,h,q,k] = sum over the four corners j of
 * grid[b,q,h,r_j,a_j] * w_j, with corners (r0,a0), (r0,a1), (r1,a0), (r1,a1)
 * and weights (1-rw)(1-aw), (1-rw)aw, rw(1-aw), rw aw taken from the (Q, Q)
 * sampling tables at (q, k); 0 where valid[q,k] is false (a corner index
 * outside 0..3 / 0..11 also counts 0).  Replaces the launch of
 * `_dense_look_grid_forward` in `_DenseLookGridSample.forward`
 * (layers/triton_dense_look_grid.py:114-150), reached through
 * `dense_look_grid_sample` (:184-202).
 *   grid  : (batch, queries, heads, 4, 12), dtype `dtype`, any strides
 *   tables: radial0, radial1, angular0, angular1 int64; radial_fraction,
 *           angular_fraction float32; valid bool (one byte); each (queries,
 *           queries) with its own (q, k) element strides, in that order
 *   out   : (batch, heads, queries, queries), dtype `dtype`, any strides
 * Arithmetic in float32, one rounding to `dtype` at the store.              */
typedef struct dlg_args {
  int64_t batch, queries, heads;
  int32_t dtype;                 /* INTP_F32 / INTP_F16 / INTP_BF16 (grid, out) */
  const void* grid;  int64_t grid_stride[5];
  const int64_t* radial0;
  const int64_t* radial1;
  const int64_t* angular0;
  const int64_t* angular1;
  const float* radial_fraction;
  const float* angular_fraction;
  const uint8_t* valid;
  int64_t table_stride[7][2];    /* (q, k) strides of the seven tables above  */
  void* out;         int64_t out_stride[4];
} dlg_args;

typedef struct dlg_grad_strides {
  int64_t stride[4];             /* (batch, heads, queries, keys) of grad_out */
} dlg_grad_strides;

INTP_API intp_status dlg_forward(const dlg_args* args, void* stream);

/* Gradient of dlg_forward with respect to the grid (the reference's
 * scatter_add backward, layers/triton_dense_look_grid.py:152-181):
 * grad_grid[b,q,h,r,a] = sum over (k, corner j) with (r_j, a_j) = (r, a) of
 * grad_out[b,h,q,k] * w_j(q, k).  grad_out has dtype args->dtype and the
 * strides `grad_strides`; grad_grid is written contiguous (batch, queries,
 * heads, 4, 12) in args->dtype.  Each cell is summed in float32 in a fixed
 * (key, corner) order, so the result is deterministic.  args->grid and
 * args->out are not used.  queries <= 1024.                                 */
INTP_API intp_status dlg_backward(const dlg_args* args, const void* grad_out, const dlg_grad_strides* grad_strides,
                                  void* grad_grid, void* stream);

/* Copies the device status word to the host (synchronous on `stream`) and
 * clears it.  *code = 0 and INTP_OK when nothing was recorded; code 0x201 (a
 * slot byte out of range in sla_forward_noalloc) returns INTP_ERR_ARGUMENT;
 * every other code is a bounded wait that gave up (INTP_ERR_TIMEOUT).        */
INTP_API intp_status sla_read_status(int32_t* status_dev, int32_t* code, void* stream);

/* Longest sequence (tokens, CLS included) sla_forward_noalloc accepts. */
#define SLA_NOALLOC_MAX_SEQ 1025

/* Look-attention forward that allocates nothing, for callers that cannot
 * allocate device memory: plugins whose enqueue step must not allocate
 * because the host framework plans all memory ahead of time, serving loops
 * that forbid allocation after start-up, and callers with a fixed memory
 * budget.  No counterpart in the reference (its Triton launch allocates its
 * outputs itself); this entry point has no reference citation for that reason.
 *
 * Same arguments as sla_forward in SLOTS mode on the tensor-core path (bf16 or
 * f16, head_dim 64), except that `slots` is the plain (Np x Np) uint8 slot
 * table in device memory (SLA_SLOT_NONE = no bias); args->slots_packed and
 * args->slot_tile_flags are ignored.  The table is packed on the GPU into a
 * library-owned file-scope __device__ scratch array of about 1.2 MB, which
 * every GPU that loads the library holds until the process exits.
 *
 * Errors: the host-side checks of sla_forward (null q / k / v / out / pose,
 * dtype codes, kernel selector, unit head_dim stride) run first and a
 * rejected call launches nothing.  Errors found on the GPU go to the int32
 * status word: args->status, a caller-owned device int32 (read it with
 * sla_read_status), receives bounded-wait failures (INTP_ERR_TIMEOUT) and a
 * slot byte >= n_slots other than SLA_SLOT_NONE (INTP_ERR_ARGUMENT; that
 * pair then gets no bias, where sla_pack_slot_table would have refused the
 * table).  When args->status is NULL these are recorded in the scratch, which
 * no call exposes: callers that need to learn of them pass a status word.
 *
 * Limits and behaviour:
 *   - seq > SLA_NOALLOC_MAX_SEQ, or a request the tensor-core path cannot
 *     take, returns INTP_ERR_UNSUPPORTED without launching anything.
 *   - The first call on each device resolves the scratch address with that
 *     device current and caches it for the process; make that first call
 *     before any stream capture, and do not use this entry point across a
 *     cudaDeviceReset (the cached address belongs to the old context).
 *   - Every call shares the scratch and leaves its contents behind; calls
 *     whose work overlaps on the GPU (several streams or threads) race.
 *   - Calls no cudaMalloc / cudaFree and no allocating library routine.      */
INTP_API intp_status sla_forward_noalloc(const sla_forward_args* args, const uint8_t* slots, void* stream);

/* Wall-clock budget (nanoseconds, 1 .. 1e9; default 1e9 = one second) of the
 * pipeline waits of the tensor-core Look-attention kernels, for the launches
 * that follow (process-wide).  A wait that runs out raises the kernel's abort
 * flag: every role stops, in-flight copies and MMAs are drained under the full
 * one-second budget, tensor memory is freed and the status word receives the
 * role's code (sla_read_status then returns INTP_ERR_TIMEOUT); the output of
 * that launch is unspecified.  A short budget makes that path testable
 * without a hung wait.                                                      */
INTP_API intp_status intp_set_wait_budget_ns(uint64_t budget_ns);

/* Library / device facts: compute capability of the current device and the
 * library's ABI version.                                                    */
INTP_API intp_status intp_device_info(int32_t* sm_major, int32_t* sm_minor, int32_t* sm_count);
INTP_API int32_t intp_abi_version(void);
INTP_API const char* intp_status_string(intp_status status);

#ifdef __cplusplus
}
#endif
#endif /* INTP_B200_H */
