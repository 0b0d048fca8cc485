// Allocation-free variant of the batched prefill forward.
//
// Some callers cannot allocate device memory at the point where they run
// attention: a plugin whose host framework owns every byte of device memory and
// hands the plugin only its input and output buffers, a serving loop that runs
// under a fixed memory budget and must not call cudaMalloc (which can also
// synchronise the device) on its hot path, or code running inside an
// allocator's own callback.  swa_prefill_forward needs a small caller-provided
// workspace, and the batched path additionally needs per-row counts and a
// validation status on the device.  This entry point keeps all of that scratch
// in one fixed array that lives in the library itself, so the caller passes
// only inputs and outputs.
#include <mutex>

#include "../../include/swattn_b200.h"
#include "swattn_internal.h"

namespace {

// Scratch shared by every call on a device (held by each GPU that loads the
// library until the process exits):
//   [0] work counter of the persistent prefill kernel (reset by every call)
//   [1] status word of the prefill kernel (device-side wait timeout)
//   [2] validation status (range / order / padding / coverage bits)
//   [3] unused
//   [4 .. 4 + 2 * B) per-row counts: full list row, then local list row
constexpr int kScratchWords = 4096;  // 16 KB
static __device__ __align__(256) int32_t g_noalloc_scratch[kScratchWords];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
int32_t* g_scratch_ptr[kMaxDevices] = {};

int fail(int code, const char* msg) {
  swa::set_last_error(msg);
  return code;
}

// Device address of the scratch array for the current device, resolved with that
// device current.  Only a successful lookup is kept: if it fails (no context yet,
// or the call came during a stream capture), the error is returned and the next
// call on that device tries again, so the failure is not sticky.
cudaError_t scratch_for_device(int dev, int32_t** out) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      *out = nullptr;
      return e;
    }
    g_scratch_ptr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int swa_noalloc_max_batch(void) { return (kScratchWords - 4) / 2; }

extern "C" int swa_prefill_forward_noalloc(const void* q, const void* k, const void* v, const int32_t* full_idx,
                                           const int32_t* local_idx, int full_stride, int local_stride,
                                           const int32_t* full_starts, const int32_t* local_starts,
                                           const int32_t* causal_ends, void* out, float* lse, int B, int Sq,
                                           int Skv, int Hq, int Hkv, int head_dim, int window, float scale_log2,
                                           int32_t* status_out, void* stream) {
  if (B <= 0 || B > swa_noalloc_max_batch()) return fail(SWA_E_INVALID, "batch size outside [1, swa_noalloc_max_batch()]");
  if (full_stride < 0 || local_stride < 0) return fail(SWA_E_INVALID, "negative index list width");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SWA_E_CUDA, "cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return fail(SWA_E_UNSUPPORTED, "device ordinal too large");
  int32_t* scratch = nullptr;
  e = scratch_for_device(dev, &scratch);
  if (e != cudaSuccess || scratch == nullptr) return fail(SWA_E_CUDA, "cudaGetSymbolAddress of the scratch array failed");

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // everything that must start at zero: counter, both status words, the counts
  e = cudaMemsetAsync(scratch, 0, sizeof(int32_t) * (4 + 2 * B), s);
  if (e != cudaSuccess) return fail(SWA_E_CUDA, "clearing the scratch array failed");
  int32_t* vstatus = scratch + 2;
  int32_t* counts = scratch + 4;
  int rc = swa_prepare_indices(full_idx, B, full_stride, Sq, 1, 0, nullptr, counts, vstatus, SWA_STATUS_FULL_RANGE,
                               SWA_STATUS_FULL_ORDER, SWA_STATUS_FULL_PAD, stream);
  if (rc != SWA_OK) return rc;
  rc = swa_prepare_indices(local_idx, B, local_stride, Sq, 1, 0, nullptr, counts + B, vstatus, SWA_STATUS_LOCAL_RANGE,
                           SWA_STATUS_LOCAL_ORDER, SWA_STATUS_LOCAL_PAD, stream);
  if (rc != SWA_OK) return rc;
  rc = swa_check_cover(counts, B, Sq, vstatus, stream);
  if (rc != SWA_OK) return rc;
  // The prefill kernel reads counts[branch * B + b], skips all work when the
  // validation status is non-zero, and uses scratch[0..1] as its workspace.
  rc = swa_prefill_forward(q, k, v, full_idx, local_idx, full_stride, local_stride, full_stride, local_stride,
                           counts, 0, 0, 0, full_starts, local_starts, causal_ends, nullptr, 0, out, lse, B, Sq, Skv, Hq,
                           Hkv, head_dim, window, scale_log2, vstatus, scratch, 16, stream);
  if (rc != SWA_OK) return rc;
  if (status_out != nullptr) {
    // status_out[0] = validation bits, status_out[1] = prefill kernel status bits,
    // for the caller to read whenever it synchronises
    e = cudaMemcpyAsync(status_out, vstatus, sizeof(int32_t), cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(status_out + 1, scratch + 1, sizeof(int32_t), cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return fail(SWA_E_CUDA, "copying the status words failed");
  }
  return SWA_OK;
}
