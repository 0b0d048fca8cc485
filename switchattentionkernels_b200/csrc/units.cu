// Unit-major <-> row-major moves of the multi-GPU driver.
//
// The sharded path gives every rank a set of (batch b, KV group g) units and
// keeps a rank's tensors unit-major: [slots, S, r * C] (r = Hq / Hkv query heads
// of the group, C elements per head: 128 for q / O, 1 for LSE), which is what
// one all-gather of every rank's outputs produces.  swa_scatter_units writes such
// slots into the row-major [B, S, Hq * C] layout of the single-GPU API (the
// permute after the all-gather); swa_gather_units is the inverse (a rank's unit
// slices of a row-major tensor).  HBM-bound byte moves: one pass, 16-byte vector
// loads and stores when a unit's row chunk allows it.
#include "../../include/swattn_b200.h"
#include "swattn_internal.h"

namespace swa {
namespace {

// One (slot, position) row chunk of `chunk_words` words of type V.  to_rows = 1:
// unit-major src -> row-major dst; 0: row-major src -> unit-major dst.  Grid:
// x over the S * chunk_words words of one slot, y over the slots.
template <typename V>
__global__ void __launch_bounds__(256) move_units_kernel(const V* __restrict__ src, V* __restrict__ dst,
                                                         const int32_t* __restrict__ unit_of_slot, int S, int hkv,
                                                         int chunk_words, int heads_words, int to_rows) {
  const int slot = blockIdx.y;
  const int u = __ldg(unit_of_slot + slot);
  if (u < 0) return;  // padding slot
  const int b = u / hkv, g = u - b * hkv;
  const uint32_t per_slot = static_cast<uint32_t>(S) * static_cast<uint32_t>(chunk_words);
  const int64_t slot_base = static_cast<int64_t>(slot) * per_slot;
  const int64_t row_base = static_cast<int64_t>(b) * S * heads_words + static_cast<int64_t>(g) * chunk_words;
  for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < per_slot; j += gridDim.x * blockDim.x) {
    const uint32_t s = j / static_cast<uint32_t>(chunk_words);
    const uint32_t w = j - s * static_cast<uint32_t>(chunk_words);
    const int64_t row = row_base + static_cast<int64_t>(s) * heads_words + w;
    if (to_rows) {
      dst[row] = src[slot_base + j];
    } else {
      dst[slot_base + j] = src[row];
    }
  }
}

cudaError_t launch_move_units(const void* src, void* dst, const int32_t* unit_of_slot, int n_slots, int S, int hkv,
                              int chunk_bytes, int row_bytes, int to_rows, cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool vec = chunk_bytes % 16 == 0 && row_bytes % 16 == 0 &&
                   (reinterpret_cast<uintptr_t>(src) & 15u) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
  const int wb = vec ? 16 : 4;
  const int64_t per_slot = static_cast<int64_t>(S) * (chunk_bytes / wb);
  // about eight resident blocks per SM over all slots
  const int64_t want_x = (per_slot + 255) / 256;
  const int64_t cap_x = (8LL * sms + n_slots - 1) / n_slots;
  const dim3 grid(static_cast<unsigned>(want_x < cap_x ? want_x : cap_x), static_cast<unsigned>(n_slots));
  if (vec) {
    move_units_kernel<uint4><<<grid, 256, 0, stream>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst),
                                                       unit_of_slot, S, hkv, chunk_bytes / 16, row_bytes / 16,
                                                       to_rows);
  } else {
    move_units_kernel<uint32_t><<<grid, 256, 0, stream>>>(static_cast<const uint32_t*>(src),
                                                          static_cast<uint32_t*>(dst), unit_of_slot, S, hkv,
                                                          chunk_bytes / 4, row_bytes / 4, to_rows);
  }
  return cudaGetLastError();
}

int check_args(const void* src, void* dst, const int32_t* unit_of_slot, int n_slots, int S, int hkv, int chunk_bytes,
               int row_bytes) {
  if (n_slots < 0 || S < 0 || hkv <= 0 || chunk_bytes <= 0 || row_bytes <= 0) {
    set_last_error("move_units: bad shape");
    return SWA_E_INVALID;
  }
  if (chunk_bytes % 4 != 0 || row_bytes % 4 != 0 || row_bytes < chunk_bytes * hkv) {
    set_last_error("move_units: chunk_bytes and row_bytes must be multiples of 4 with row_bytes >= hkv * chunk_bytes");
    return SWA_E_INVALID;
  }
  if (n_slots > 65535 || static_cast<int64_t>(S) * (chunk_bytes / 4) >= (1LL << 31)) {
    set_last_error("move_units: at most 65535 slots and 2^31 words per slot");
    return SWA_E_INVALID;
  }
  if (n_slots > 0 && S > 0 && (src == nullptr || dst == nullptr || unit_of_slot == nullptr)) {
    set_last_error("move_units: null pointer");
    return SWA_E_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(src) & 3u) != 0 || (reinterpret_cast<uintptr_t>(dst) & 3u) != 0) {
    set_last_error("move_units: pointers must be 4-byte aligned");
    return SWA_E_INVALID;
  }
  return SWA_OK;
}

struct BroadcastDsts {
  uint4* p[8];
  int n;
};

// Each 16-byte word of src is loaded once and stored to every destination (this
// GPU's memory or a peer's over NVLink: plain st.global).
__global__ void __launch_bounds__(256) broadcast_kernel(const uint4* __restrict__ src, size_t words, BroadcastDsts d) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < words;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint4 v = src[i];
    for (int t = 0; t < d.n; ++t) d.p[t][i] = v;
  }
}

}  // namespace
}  // namespace swa

extern "C" int swa_broadcast_bytes(const void* src, size_t bytes, void* const* dsts, int n_dst, void* stream) {
  if (n_dst < 0 || n_dst > 8 || (n_dst > 0 && dsts == nullptr)) {
    swa::set_last_error("broadcast_bytes: 0 to 8 destinations");
    return SWA_E_INVALID;
  }
  if (bytes == 0 || n_dst == 0) return SWA_OK;
  if (src == nullptr || bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(src) & 15u) != 0) {
    swa::set_last_error("broadcast_bytes: src and bytes must be multiples of 16");
    return SWA_E_INVALID;
  }
  swa::BroadcastDsts d{};
  d.n = n_dst;
  for (int i = 0; i < n_dst; ++i) {
    if (dsts[i] == nullptr || (reinterpret_cast<uintptr_t>(dsts[i]) & 15u) != 0) {
      swa::set_last_error("broadcast_bytes: destinations must be non-null and 16-byte aligned");
      return SWA_E_INVALID;
    }
    d.p[i] = static_cast<uint4*>(dsts[i]);
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t words = bytes / 16;
  const size_t want = (words + 255) / 256;
  const unsigned blocks = static_cast<unsigned>(want < static_cast<size_t>(8 * sms) ? want : static_cast<size_t>(8 * sms));
  swa::broadcast_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint4*>(src), words,
                                                                              d);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    swa::set_last_error(cudaGetErrorString(e));
    return SWA_E_CUDA;
  }
  return SWA_OK;
}

extern "C" int swa_scatter_units(const void* src, const int32_t* unit_of_slot, int n_slots, int S, int hkv,
                                 int chunk_bytes, int row_bytes, void* dst, void* stream) {
  const int rc = swa::check_args(src, dst, unit_of_slot, n_slots, S, hkv, chunk_bytes, row_bytes);
  if (rc != SWA_OK) return rc;
  if (n_slots == 0 || S == 0) return SWA_OK;
  const cudaError_t e = swa::launch_move_units(src, dst, unit_of_slot, n_slots, S, hkv, chunk_bytes, row_bytes, 1,
                                               static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    swa::set_last_error(cudaGetErrorString(e));
    return SWA_E_CUDA;
  }
  return SWA_OK;
}

extern "C" int swa_gather_units(const void* src, const int32_t* unit_of_slot, int n_slots, int S, int hkv,
                                int chunk_bytes, int row_bytes, void* dst, void* stream) {
  const int rc = swa::check_args(src, dst, unit_of_slot, n_slots, S, hkv, chunk_bytes, row_bytes);
  if (rc != SWA_OK) return rc;
  if (n_slots == 0 || S == 0) return SWA_OK;
  const cudaError_t e = swa::launch_move_units(src, dst, unit_of_slot, n_slots, S, hkv, chunk_bytes, row_bytes, 0,
                                               static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    swa::set_last_error(cudaGetErrorString(e));
    return SWA_E_CUDA;
  }
  return SWA_OK;
}
