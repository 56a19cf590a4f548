// noalloc.cu - Look-attention forward for callers that cannot allocate device memory.
//
// sla_forward needs two device buffers besides the tensors themselves: the
// packed slot table (built on the host by sla_pack_slot_table and uploaded by
// the caller) and a status word for the kernel's bounded waits.  Some callers
// cannot allocate device memory for them: plugins whose enqueue step must not
// allocate because the host framework plans all memory ahead of time, serving
// loops that forbid allocation after start-up, and embedded callers with a
// fixed device-memory budget.  sla_forward_noalloc serves those callers: it
// takes the plain (Np x Np) slot table as an ordinary device input, packs it on
// the GPU into a scratch area that the library owns as a file-scope __device__
// array, and runs the same tensor-core kernel.  It calls no cudaMalloc or
// cudaFree and no allocating library routine.
//
// The scratch array is sized for sequences up to SLA_NOALLOC_MAX_SEQ tokens
// (1025: CLS + a 32 x 32 lattice): 9 x 17 tiles of 8 KB plus flags and the
// status word, about 1.2 MB.  Every GPU that loads the library holds it until
// the process exits.
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include <mutex>
#include "../../include/intp_b200.h"
#include "sla_internal.h"

namespace {

constexpr int64_t kMaxSeq = SLA_NOALLOC_MAX_SEQ;
constexpr int64_t kMaxQTiles = (kMaxSeq + intp::kSlotTileQ - 1) / intp::kSlotTileQ;  // 9
constexpr int64_t kMaxKTiles = (kMaxSeq + intp::kSlotTileK - 1) / intp::kSlotTileK;  // 17
constexpr int64_t kPackedBytes = kMaxQTiles * kMaxKTiles * intp::kSlotTileBytes;    // 1,253,376
constexpr int64_t kFlagsOffset = kPackedBytes;
constexpr int64_t kStatusOffset = kFlagsOffset + 256;  // flags need kMaxQTiles * kMaxKTiles = 153 bytes
constexpr int64_t kScratchBytes = kStatusOffset + 256;
static_assert(kMaxQTiles * kMaxKTiles <= 256, "flag area too small");
// Status-word code of a slot byte >= n_slots that is not SLA_SLOT_NONE.
constexpr int32_t kDevBadSlot = 0x201;

// The library-owned scratch.  In host code `g_scratch` is only a host-side
// stand-in for the symbol: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_scratch[kScratchBytes];

struct DeviceScratch {
  uint8_t* base = nullptr;
  int sms = 0;
  bool ready = false;
};

std::mutex g_mu;
DeviceScratch g_devices[64];

// Per-device set-up on the first call: resolve the scratch address with the
// device current and cache it.  Returns nullptr on failure.
const DeviceScratch* scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceScratch& d = g_devices[dev];
  if (!d.ready) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_scratch) != cudaSuccess || ptr == nullptr) return nullptr;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return nullptr;
    if (prop.major != 10) return nullptr;
    d.base = static_cast<uint8_t*>(ptr);
    d.sms = prop.multiProcessorCount;
    d.ready = true;
  }
  return &d;
}

// Packs a patch-indexed (Np x Np) slot table into the token-indexed tile layout
// of sla_pack_slot_table (token i = patch i-1; CLS row/column, padding rows and
// SLA_SLOT_NONE become n_slots, key columns past the end n_slots + 1) and
// writes one "needs lookup" flag per tile.  One
// thread block per tile; every byte of the used tiles and flags is written.
__global__ void pack_slots_kernel(const uint8_t* __restrict__ slots, int64_t patch_count, int32_t n_slots,
                                  int64_t n_kt, uint8_t* __restrict__ packed, uint8_t* __restrict__ flags,
                                  int32_t* status) {
  const int64_t tile = blockIdx.x;
  const int64_t qt = tile / n_kt, kt = tile % n_kt;
  uint8_t* dst = packed + tile * intp::kSlotTileBytes;
  __shared__ uint32_t bits;  // bit w: rows 32w..32w+31 of the tile need the lookup
  if (threadIdx.x == 0) bits = 0;
  __syncthreads();
  uint32_t mine = 0;
  for (int e = threadIdx.x; e < intp::kSlotTileBytes; e += blockDim.x) {
    const int chunk = e / 2048, r = (e % 2048) / 16, c16 = e % 16;
    const int64_t i = qt * intp::kSlotTileQ + r;           // query token
    const int64_t j = kt * intp::kSlotTileK + chunk * 16 + c16;  // key token
    uint8_t v = static_cast<uint8_t>(n_slots);
    if (j > patch_count) {
      v = static_cast<uint8_t>(n_slots + 1);  // key past the sequence end: looked up as -inf
      mine |= 0xFu;
    } else if (i >= 1 && j >= 1 && i <= patch_count) {
      const uint8_t s = slots[(i - 1) * patch_count + (j - 1)];
      if (s != SLA_SLOT_NONE && s < n_slots) {
        v = s;
        mine |= 1u << (r / 32);
      } else if (s != SLA_SLOT_NONE) {
        // sla_pack_slot_table rejects this byte; here the pair gets no bias
        // and the status word says so (sla_read_status: INTP_ERR_ARGUMENT).
        atomicCAS(status, 0, kDevBadSlot);
      }
    }
    dst[e] = v;
  }
  if (mine) atomicOr(&bits, mine);
  __syncthreads();
  if (threadIdx.x == 0) flags[tile] = static_cast<uint8_t>(bits);
}

}  // namespace

extern "C" INTP_API intp_status sla_forward_noalloc(const sla_forward_args* a, const uint8_t* slots, void* stream) {
  // The checks sla_forward makes, in its order, before anything is looked up
  // or launched: a rejected call touches no device memory.
  if (!a || !slots) return INTP_ERR_ARGUMENT;
  if (a->batch < 0 || a->heads < 0 || a->seq < 2 || a->head_dim < 1) return INTP_ERR_SHAPE;
  if (a->dtype != INTP_F32 && a->dtype != INTP_F16 && a->dtype != INTP_BF16) return INTP_ERR_DTYPE;
  if (a->kernel < SLA_KERNEL_AUTO || a->kernel > SLA_KERNEL_TCGEN05) return INTP_ERR_ARGUMENT;
  if (a->bias_mode != SLA_BIAS_SLOTS || a->dense != nullptr || a->kernel == SLA_KERNEL_SIMT)
    return INTP_ERR_UNSUPPORTED;
  if (a->seq > kMaxSeq) return INTP_ERR_UNSUPPORTED;  // beyond the scratch capacity
  if (a->batch == 0 || a->heads == 0) return INTP_OK;
  if (!a->q || !a->k || !a->v || !a->out || !a->pose) return INTP_ERR_ARGUMENT;
  if (a->poses < 1 || a->poses > 253) return INTP_ERR_ARGUMENT;
  if (a->pose_dtype != INTP_F32 && a->pose_dtype != INTP_F16 && a->pose_dtype != INTP_BF16) return INTP_ERR_DTYPE;
  if (a->q_stride[3] != 1 || a->k_stride[3] != 1 || a->v_stride[3] != 1 || a->out_stride[3] != 1)
    return INTP_ERR_LAYOUT;
  const DeviceScratch* d = scratch_for_current_device();
  if (!d) return INTP_ERR_ARCH;

  intp::SlaParams p;
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
  p.bias_mode = SLA_BIAS_SLOTS;
  p.poses = a->poses;
  p.pose = a->pose;
  std::memcpy(p.pose_stride, a->pose_stride, sizeof(p.pose_stride));
  p.pose_dtype = a->pose_dtype;
  p.slots_packed = d->base;
  p.slot_tile_flags = d->base + kFlagsOffset;
  // A caller-provided status word (an output the caller owns) receives
  // bounded-wait failures; without one they land in the scratch word.
  p.status = a->status ? a->status : reinterpret_cast<int32_t*>(d->base + kStatusOffset);
  if (!intp::sla_tc_supported(p)) return INTP_ERR_UNSUPPORTED;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t patch_count = a->seq - 1;
  const int64_t n_qt = (a->seq + intp::kSlotTileQ - 1) / intp::kSlotTileQ;
  const int64_t n_kt = (a->seq + intp::kSlotTileK - 1) / intp::kSlotTileK;
  // The scratch status word must start at zero; the packed tiles and flags are
  // fully rewritten below.  Scratch contents persist between calls, so calls
  // whose work overlaps on the GPU (other streams, other threads) race on it.
  if (cudaMemsetAsync(d->base + kStatusOffset, 0, sizeof(int32_t), s) != cudaSuccess) return INTP_ERR_LAUNCH;
  pack_slots_kernel<<<static_cast<unsigned>(n_qt * n_kt), 256, 0, s>>>(
      slots, patch_count, static_cast<int32_t>(a->poses), n_kt, d->base, d->base + kFlagsOffset, p.status);
  if (cudaGetLastError() != cudaSuccess) return INTP_ERR_LAUNCH;
  return intp::launch_sla_tc(p, s, d->sms);
}
