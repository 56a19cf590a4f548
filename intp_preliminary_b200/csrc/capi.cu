// capi.cu - extern "C" boundary of libintp_b200.so (declared in include/intp_b200.h).
//
// Validates arguments with the same rules as the reference's Python launch
// sites, picks the kernel, launches on the caller's stream, and maps every
// failure to an intp_status.  No exception crosses this boundary and nothing
// here allocates device memory.
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include <atomic>
#include <mutex>
#include "../../include/intp_b200.h"
#include "sla_internal.h"

namespace {

struct DeviceFacts {
  int major = 0, minor = 0, sms = 0;
};

bool device_facts(DeviceFacts* f) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  static std::mutex mu;
  static DeviceFacts cache[64];
  static bool have[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && have[dev]) {
    *f = cache[dev];
    return true;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return false;
  f->major = prop.major;
  f->minor = prop.minor;
  f->sms = prop.multiProcessorCount;
  if (dev >= 0 && dev < 64) {
    cache[dev] = *f;
    have[dev] = true;
  }
  return true;
}

bool valid_dtype(int32_t d) { return d == INTP_F32 || d == INTP_F16 || d == INTP_BF16; }

std::atomic<uint64_t> g_wait_budget_ns{1000000000ull};

}  // namespace

namespace intp {
uint64_t tc_wait_budget_ns() { return g_wait_budget_ns.load(std::memory_order_relaxed); }
}  // namespace intp

extern "C" {

int32_t intp_abi_version(void) { return 3; }

const char* intp_status_string(intp_status s) {
  switch (s) {
    case INTP_OK: return "ok";
    case INTP_ERR_ARGUMENT: return "invalid argument";
    case INTP_ERR_SHAPE: return "shape mismatch";
    case INTP_ERR_DTYPE: return "unsupported dtype";
    case INTP_ERR_LAYOUT: return "unsupported stride or alignment";
    case INTP_ERR_ARCH: return "device is not sm_100 (B200)";
    case INTP_ERR_LAUNCH: return "CUDA launch failure";
    case INTP_ERR_TIMEOUT: return "a bounded device wait timed out";
    case INTP_ERR_UNSUPPORTED: return "request outside kernel coverage";
    default: return "unknown status";
  }
}

intp_status intp_set_wait_budget_ns(uint64_t budget_ns) {
  if (budget_ns == 0 || budget_ns > 1000000000ull) return INTP_ERR_ARGUMENT;
  g_wait_budget_ns.store(budget_ns, std::memory_order_relaxed);
  return INTP_OK;
}

intp_status intp_device_info(int32_t* sm_major, int32_t* sm_minor, int32_t* sm_count) {
  DeviceFacts f;
  if (!device_facts(&f)) return INTP_ERR_LAUNCH;
  if (sm_major) *sm_major = f.major;
  if (sm_minor) *sm_minor = f.minor;
  if (sm_count) *sm_count = f.sms;
  return INTP_OK;
}

intp_status sla_slot_table_bytes(int64_t seq, int64_t* packed_bytes, int64_t* flag_bytes) {
  if (seq < 1 || !packed_bytes || !flag_bytes) return INTP_ERR_ARGUMENT;
  const int64_t nqt = (seq + intp::kSlotTileQ - 1) / intp::kSlotTileQ;
  const int64_t nkt = (seq + intp::kSlotTileK - 1) / intp::kSlotTileK;
  *packed_bytes = nqt * nkt * intp::kSlotTileBytes;
  *flag_bytes = nqt * nkt;
  return INTP_OK;
}

// Packs a patch-indexed (Np x Np) slot table into token-indexed tiles: token i
// = patch i-1; token 0 (CLS), unslotted pairs and padding query rows carry
// n_slots ("no bias"); key columns past the sequence end carry n_slots + 1
// ("padding key", looked up as -inf so the kernel needs no per-key mask).
intp_status sla_pack_slot_table(const uint8_t* slots, int64_t patch_count, int32_t n_slots, uint8_t* packed,
                                uint8_t* tile_flags) {
  if (!slots || !packed || !tile_flags || patch_count < 0) return INTP_ERR_ARGUMENT;
  if (n_slots < 1 || n_slots > 253) return INTP_ERR_ARGUMENT;
  const int64_t seq = patch_count + 1;
  int64_t pb = 0, fb = 0;
  sla_slot_table_bytes(seq, &pb, &fb);
  const int64_t nkt = (seq + intp::kSlotTileK - 1) / intp::kSlotTileK;
  std::memset(packed, n_slots, static_cast<size_t>(pb));
  std::memset(tile_flags, 0, static_cast<size_t>(fb));
  for (int64_t pq = 0; pq < patch_count; ++pq) {
    const int64_t i = pq + 1;
    const int64_t qt = i / intp::kSlotTileQ, r = i % intp::kSlotTileQ;
    for (int64_t pk = 0; pk < patch_count; ++pk) {
      const uint8_t s = slots[pq * patch_count + pk];
      if (s == SLA_SLOT_NONE) continue;
      if (s >= n_slots) return INTP_ERR_ARGUMENT;
      const int64_t j = pk + 1;
      const int64_t kt = j / intp::kSlotTileK, c = j % intp::kSlotTileK;
      const int64_t off = (qt * nkt + kt) * intp::kSlotTileBytes + (c / 16) * 2048 + r * 16 + (c % 16);
      packed[off] = s;
      tile_flags[qt * nkt + kt] |= static_cast<uint8_t>(1u << (r / 32));  // bit w: rows 32w..32w+31
    }
  }
  if (seq % intp::kSlotTileK != 0) {
    const int64_t nqt = (seq + intp::kSlotTileQ - 1) / intp::kSlotTileQ;
    const int64_t kt = nkt - 1;
    for (int64_t qt = 0; qt < nqt; ++qt) {
      for (int64_t c = seq % intp::kSlotTileK; c < intp::kSlotTileK; ++c)
        for (int64_t r = 0; r < intp::kSlotTileQ; ++r)
          packed[(qt * nkt + kt) * intp::kSlotTileBytes + (c / 16) * 2048 + r * 16 + (c % 16)] =
              static_cast<uint8_t>(n_slots + 1);
      tile_flags[qt * nkt + kt] |= 0xF;  // every row sees the masked keys
    }
  }
  return INTP_OK;
}

}  // extern "C"

namespace {

// Validates forward arguments (the reference's launch-site rules) and fills the
// kernel parameter block.  INTP_OK with *empty set means there is no work.
intp_status to_params(const sla_forward_args* a, intp::SlaParams* out, bool* empty) {
  *empty = false;
  if (!a) return INTP_ERR_ARGUMENT;
  if (a->batch < 0 || a->heads < 0 || a->seq < 1 || a->head_dim < 1) return INTP_ERR_SHAPE;
  if (!valid_dtype(a->dtype)) return INTP_ERR_DTYPE;
  if (a->batch == 0 || a->heads == 0) {
    *empty = true;
    return INTP_OK;
  }
  if (!a->q || !a->k || !a->v || !a->out) return INTP_ERR_ARGUMENT;
  if (a->q_stride[3] != 1 || a->k_stride[3] != 1 || a->v_stride[3] != 1 || a->out_stride[3] != 1)
    return INTP_ERR_LAYOUT;
  if (a->bias_mode == SLA_BIAS_FIELDS) {
    if (!a->pose || !a->fields || a->poses < 1) return INTP_ERR_ARGUMENT;
    if (!valid_dtype(a->pose_dtype) || !valid_dtype(a->fields_dtype)) return INTP_ERR_DTYPE;
  } else if (a->bias_mode == SLA_BIAS_SLOTS) {
    if (!a->pose || !a->slots_packed || !a->slot_tile_flags || a->poses < 1 || a->poses > 253)
      return INTP_ERR_ARGUMENT;
    if (!valid_dtype(a->pose_dtype)) return INTP_ERR_DTYPE;
  } else if (a->bias_mode == SLA_BIAS_SLOT_FIELDS) {
    if (!a->pose || !a->fields || !a->slots_packed || !a->slot_tile_flags || a->poses < 1 || a->slots < 1 ||
        a->slots > 253)
      return INTP_ERR_ARGUMENT;
    if (!valid_dtype(a->pose_dtype) || !valid_dtype(a->fields_dtype)) return INTP_ERR_DTYPE;
  } else if (a->bias_mode != SLA_BIAS_NONE) {
    return INTP_ERR_ARGUMENT;
  }
  if (a->dense && !valid_dtype(a->dense_dtype)) return INTP_ERR_DTYPE;
  if (a->kernel < SLA_KERNEL_AUTO || a->kernel > SLA_KERNEL_TCGEN05) return INTP_ERR_ARGUMENT;

  intp::SlaParams& p = *out;
  std::memset(&p, 0, sizeof(p));
  p.batch = a->batch;
  p.heads = a->heads;
  p.seq = a->seq;
  p.head_dim = a->head_dim;
  p.scale = a->scale;
  p.dtype = a->dtype;
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.out = a->out;
  std::memcpy(p.q_stride, a->q_stride, sizeof(p.q_stride));
  std::memcpy(p.k_stride, a->k_stride, sizeof(p.k_stride));
  std::memcpy(p.v_stride, a->v_stride, sizeof(p.v_stride));
  std::memcpy(p.out_stride, a->out_stride, sizeof(p.out_stride));
  p.lse = a->lse;
  p.bias_mode = a->bias_mode;
  p.poses = a->poses;
  p.slots = a->bias_mode == SLA_BIAS_SLOT_FIELDS ? a->slots : 0;
  p.pose = a->pose;
  std::memcpy(p.pose_stride, a->pose_stride, sizeof(p.pose_stride));
  p.pose_dtype = a->pose_dtype;
  p.fields = a->fields;
  std::memcpy(p.fields_stride, a->fields_stride, sizeof(p.fields_stride));
  p.fields_dtype = a->fields_dtype;
  p.slots_packed = a->slots_packed;
  p.slot_tile_flags = a->slot_tile_flags;
  p.dense = a->dense;
  std::memcpy(p.dense_stride, a->dense_stride, sizeof(p.dense_stride));
  p.dense_dtype = a->dense_dtype;
  p.status = a->status;
  return INTP_OK;
}

}  // namespace

extern "C" {

intp_status sla_forward(const sla_forward_args* a, void* stream) {
  intp::SlaParams p;
  bool empty = false;
  const intp_status st = to_params(a, &p, &empty);
  if (st != INTP_OK || empty) return st;
  DeviceFacts f;
  if (!device_facts(&f)) return INTP_ERR_LAUNCH;
  if (f.major != 10) return INTP_ERR_ARCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->kernel != SLA_KERNEL_SIMT && intp::sla_tc_supported(p)) return intp::launch_sla_tc(p, s, f.sms);
  if (a->kernel == SLA_KERNEL_TCGEN05) return INTP_ERR_UNSUPPORTED;
  return intp::launch_sla_simt(p, s);
}

intp_status sla_backward(const sla_backward_args* a, void* stream) {
  if (!a) return INTP_ERR_ARGUMENT;
  intp::SlaBwdParams bp;
  std::memset(&bp, 0, sizeof(bp));
  bool empty = false;
  const intp_status st = to_params(&a->fwd, &bp.f, &empty);
  if (st != INTP_OK || empty) return st;
  if (!a->fwd.lse || !a->grad_out || !a->delta) return INTP_ERR_ARGUMENT;
  // SLOT_FIELDS gradients go through the SLOTS form with the per-slot values
  // pose . slot_fields materialised by the caller.
  if (a->fwd.bias_mode == SLA_BIAS_SLOT_FIELDS) return INTP_ERR_UNSUPPORTED;
  if (a->grad_fields && a->fwd.bias_mode != SLA_BIAS_FIELDS) return INTP_ERR_ARGUMENT;
  if (a->grad_pose && a->fwd.bias_mode == SLA_BIAS_NONE) return INTP_ERR_ARGUMENT;
  if (a->grad_dense && !a->fwd.dense) return INTP_ERR_ARGUMENT;
  if (a->fwd.seq < 2 && (a->grad_pose || a->grad_fields || a->grad_dense)) return INTP_ERR_SHAPE;
  DeviceFacts f;
  if (!device_facts(&f)) return INTP_ERR_LAUNCH;
  if (f.major != 10) return INTP_ERR_ARCH;
  bp.grad_out = a->grad_out;
  std::memcpy(bp.grad_out_stride, a->grad_out_stride, sizeof(bp.grad_out_stride));
  bp.grad_q = a->grad_q;
  bp.grad_k = a->grad_k;
  bp.grad_v = a->grad_v;
  bp.grad_pose = a->grad_pose;
  bp.grad_fields = a->grad_fields;
  bp.grad_dense = a->grad_dense;
  bp.delta = a->delta;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->fwd.kernel != SLA_KERNEL_SIMT && intp::sla_backward_fused_supported(bp, a->slots_packed_t))
    return intp::launch_sla_backward_fused(bp, a->slots_packed_t, s);
  if (a->fwd.kernel == SLA_KERNEL_TCGEN05) return INTP_ERR_UNSUPPORTED;
  return intp::launch_sla_backward(bp, s);
}

intp_status sla_probability_score_grad(const sla_probability_score_grad_args* a, void* stream) {
  if (!a) return INTP_ERR_ARGUMENT;
  intp::SlaParams p;
  bool empty = false;
  const intp_status st = to_params(&a->fwd, &p, &empty);
  if (st != INTP_OK || empty) return st;
  if (!a->fwd.lse || !a->grad_out || !a->probability || !a->score_grad) return INTP_ERR_ARGUMENT;
  if (a->grad_pose && a->fwd.bias_mode != SLA_BIAS_SLOTS) return INTP_ERR_ARGUMENT;
  if (a->grad_out_stride[3] != 1) return INTP_ERR_LAYOUT;
  if (a->ld < a->fwd.seq || a->ld % 8 || reinterpret_cast<uintptr_t>(a->probability) % 16 ||
      reinterpret_cast<uintptr_t>(a->score_grad) % 16)
    return INTP_ERR_LAYOUT;
  DeviceFacts f;
  if (!device_facts(&f)) return INTP_ERR_LAUNCH;
  if (f.major != 10) return INTP_ERR_ARCH;
  return intp::launch_sla_probability_score_grad(p, a->grad_out, a->grad_out_stride, a->probability, a->score_grad,
                                                 a->ld, a->grad_pose, static_cast<cudaStream_t>(stream));
}

intp_status nl1_forward(const float* x, const float* w, float* out, int64_t rows, int64_t protos, int64_t features,
                        void* stream) {
  if (rows < 0 || protos < 0 || features < 0) return INTP_ERR_SHAPE;
  if (rows == 0 || protos == 0) return INTP_OK;
  if (!out || (features > 0 && (!x || !w))) return INTP_ERR_ARGUMENT;
  DeviceFacts f;
  if (!device_facts(&f)) return INTP_ERR_LAUNCH;
  if (f.major != 10) return INTP_ERR_ARCH;
  return intp::launch_nl1(x, w, out, rows, protos, features, static_cast<cudaStream_t>(stream));
}

intp_status nl1_backward(const float* x, const float* w, const float* grad_out, float* grad_x, float* grad_w,
                         int64_t rows, int64_t protos, int64_t features, void* stream) {
  if (rows < 0 || protos < 0 || features < 0) return INTP_ERR_SHAPE;
  if (rows == 0 || protos == 0 || features == 0) return INTP_OK;
  if (!x || !w || !grad_out || (!grad_x && !grad_w)) return INTP_ERR_ARGUMENT;
  DeviceFacts f;
  if (!device_facts(&f)) return INTP_ERR_LAUNCH;
  if (f.major != 10) return INTP_ERR_ARCH;
  return intp::launch_nl1_backward(x, w, grad_out, grad_x, grad_w, rows, protos, features,
                                   static_cast<cudaStream_t>(stream));
}

intp_status sla_read_status(int32_t* status_dev, int32_t* code, void* stream) {
  if (!status_dev || !code) return INTP_ERR_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t host = 0;
  if (cudaMemcpyAsync(&host, status_dev, sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return INTP_ERR_LAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return INTP_ERR_LAUNCH;
  *code = host;
  if (host != 0) {
    if (cudaMemsetAsync(status_dev, 0, sizeof(int32_t), s) != cudaSuccess) return INTP_ERR_LAUNCH;
    // 0x201: sla_forward_noalloc met a slot byte >= n_slots (not SLA_SLOT_NONE);
    // every other code is a bounded wait that gave up.
    return host == 0x201 ? INTP_ERR_ARGUMENT : INTP_ERR_TIMEOUT;
  }
  return INTP_OK;
}

}  // extern "C"
