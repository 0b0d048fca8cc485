// C ABI of libswattn_b200 (declared in include/swattn_b200.h).
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <string>

#include "../../include/swattn_b200.h"
#include "swattn_internal.h"
#include "tma_host.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SWA_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// failure-detection test hook (swa_test_withhold_kv_load)
std::atomic<int> g_test_withhold{0};

}  // namespace

namespace swa {
void set_last_error(const char* msg) { g_last_error = msg; }
}  // namespace swa

extern "C" {

int swa_abi_version(void) { return 1; }

void swa_test_withhold_kv_load(int on) { g_test_withhold.store(on != 0 ? 1 : 0); }

const char* swa_last_error_string(void) { return g_last_error.c_str(); }

int swa_num_sms(int device) {
  int n = 0;
  cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  return n;
}

int swa_compact_mask(const uint8_t* mask, int B, int S, int32_t* full, int32_t* local, int32_t* counts,
                     void* stream) {
  if (B < 0 || S < 0) return fail(SWA_E_INVALID, "negative shape");
  if (B == 0) return SWA_OK;
  if (mask == nullptr || full == nullptr || local == nullptr || counts == nullptr)
    return fail(SWA_E_INVALID, "null pointer");
  cudaError_t e = swa::launch_compact_mask(mask, B, S, full, local, counts, nullptr, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "compact_mask launch");
  return SWA_OK;
}

static_assert(swa::kRouterBf16 == SWA_ROUTER_BF16 && swa::kRouterF32 == SWA_ROUTER_F32, "router dtype codes");

int swa_compact_router(const void* router, int dtype, int pair, float threshold, int B, int S, int32_t* full,
                       int32_t* local, int32_t* counts, void* stream) {
  if (B < 0 || S < 0) return fail(SWA_E_INVALID, "negative shape");
  if (dtype != SWA_ROUTER_BF16 && dtype != SWA_ROUTER_F32) return fail(SWA_E_INVALID, "router dtype must be bf16 or fp32");
  if (pair != 0 && pair != 1) return fail(SWA_E_INVALID, "pair must be 0 or 1");
  if (B == 0) return SWA_OK;
  if (router == nullptr || full == nullptr || local == nullptr || counts == nullptr)
    return fail(SWA_E_INVALID, "null pointer");
  cudaError_t e = swa::launch_compact_router(router, dtype, pair, threshold, B, S, full, local, counts, nullptr,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "compact_router launch");
  return SWA_OK;
}

int64_t swa_compact_workspace_elems(int B, int S) { return swa::compact_workspace_elems(B, S); }

int swa_compact_mask_ws(const uint8_t* mask, int B, int S, int32_t* full, int32_t* local, int32_t* counts,
                        int32_t* workspace, int64_t workspace_elems, void* stream) {
  if (B < 0 || S < 0) return fail(SWA_E_INVALID, "negative shape");
  if (B == 0) return SWA_OK;
  if (mask == nullptr || full == nullptr || local == nullptr || counts == nullptr)
    return fail(SWA_E_INVALID, "null pointer");
  const int64_t need = swa::compact_workspace_elems(B, S);
  if (need > 0 && (workspace == nullptr || workspace_elems < need)) return fail(SWA_E_INVALID, "workspace too small");
  cudaError_t e = swa::launch_compact_mask(mask, B, S, full, local, counts, need > 0 ? workspace : nullptr,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "compact_mask launch");
  return SWA_OK;
}

int swa_compact_router_ws(const void* router, int dtype, int pair, float threshold, int B, int S, int32_t* full,
                          int32_t* local, int32_t* counts, int32_t* workspace, int64_t workspace_elems,
                          void* stream) {
  if (B < 0 || S < 0) return fail(SWA_E_INVALID, "negative shape");
  if (dtype != SWA_ROUTER_BF16 && dtype != SWA_ROUTER_F32) return fail(SWA_E_INVALID, "router dtype must be bf16 or fp32");
  if (pair != 0 && pair != 1) return fail(SWA_E_INVALID, "pair must be 0 or 1");
  if (B == 0) return SWA_OK;
  if (router == nullptr || full == nullptr || local == nullptr || counts == nullptr)
    return fail(SWA_E_INVALID, "null pointer");
  const int64_t need = swa::compact_workspace_elems(B, S);
  if (need > 0 && (workspace == nullptr || workspace_elems < need)) return fail(SWA_E_INVALID, "workspace too small");
  cudaError_t e = swa::launch_compact_router(router, dtype, pair, threshold, B, S, full, local, counts,
                                             need > 0 ? workspace : nullptr, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "compact_router launch");
  return SWA_OK;
}

int swa_prepare_indices(const int32_t* idx, int B, int N, int seq_len, int trailing_pad, int cap,
                        int32_t* padded, int32_t* count, int32_t* status, int range_bit, int order_bit,
                        int pad_bit, void* stream) {
  if (B < 0 || N < 0 || cap < 0) return fail(SWA_E_INVALID, "negative shape");
  if (B == 0) return SWA_OK;
  if ((N > 0 && idx == nullptr) || count == nullptr || status == nullptr)
    return fail(SWA_E_INVALID, "null pointer");
  if (padded != nullptr && cap < N) return fail(SWA_E_INVALID, "capacity below list length");
  if (trailing_pad && pad_bit == 0) return fail(SWA_E_INVALID, "trailing padding needs a pad status bit");
  cudaError_t e = swa::launch_prepare_indices(idx, B, N, seq_len, B, padded ? cap : 0, padded, count, status,
                                              range_bit, order_bit, trailing_pad ? pad_bit : 0,
                                              static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "prepare_indices launch");
  return SWA_OK;
}

int swa_check_cover(const int32_t* counts, int B, int seq_len, int32_t* status, void* stream) {
  if (B <= 0) return SWA_OK;
  if (counts == nullptr || status == nullptr) return fail(SWA_E_INVALID, "null pointer");
  cudaError_t e = swa::launch_check_cover(counts, B, seq_len, status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "check_cover launch");
  return SWA_OK;
}

int swa_build_metadata(const int32_t* cu_seqlens, int nseg, int q_len, int kv_len, int window,
                       int32_t* q_positions, int32_t* kv_positions, int32_t* q_segment_ids,
                       int32_t* kv_segment_ids, int32_t* full_starts, int32_t* local_starts,
                       int32_t* causal_ends, void* stream) {
  if (q_len < 0 || kv_len < 0 || window <= 0) return fail(SWA_E_INVALID, "bad metadata shape");
  if (cu_seqlens != nullptr && (nseg <= 0 || kv_len != q_len))
    return fail(SWA_E_INVALID, "packed metadata needs nseg > 0 and kv_len == q_len");
  if (q_len == 0 && kv_len == 0) return SWA_OK;
  cudaError_t e = swa::launch_build_metadata(cu_seqlens, nseg, q_len, kv_len, window, q_positions, kv_positions,
                                             q_segment_ids, kv_segment_ids, full_starts, local_starts, causal_ends,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "build_metadata launch");
  return SWA_OK;
}

namespace {

// Split of the decode step's key axis.  Which sequences attend to all their
// keys is device data, so splits are sized for the longest possible range
// (Smax): about four waves of CTAs over the SMs if every range were full,
// clamped to 256..2048 keys (a multiple of 64) so that a long full-attention
// sequence is spread over many CTAs instead of forming the tail; splits past a
// sequence's range exit at once.
struct DecodeSplit {
  int nhb, splits, split_keys;
};

// Largest split: on the 64-sequence decode batch (16K-32K keys, p_full 0.125)
// caps of 512, 1024, 4096 and 8192 keys were all slower than 2048, for the BF16
// and for the FP8 cache.
constexpr int64_t kDecodeMaxSplitKeys = 2048;

DecodeSplit decode_split(int B, int Smax, int Hq, int Hkv, int num_sms) {
  DecodeSplit d{};
  const int r = Hq / Hkv;
  d.nhb = (r + 15) / 16;
  const int64_t units = static_cast<int64_t>(B) * Hkv * d.nhb;
  int64_t sk = (static_cast<int64_t>(Smax) * units + 4LL * num_sms - 1) / (4LL * num_sms);
  sk = (sk + 63) / 64 * 64;
  sk = std::min<int64_t>(std::max<int64_t>(sk, 256), kDecodeMaxSplitKeys);
  sk = std::min<int64_t>(sk, (static_cast<int64_t>(Smax) + 63) / 64 * 64);
  d.split_keys = static_cast<int>(sk);
  d.splits = (Smax + d.split_keys - 1) / d.split_keys;
  return d;
}

size_t decode_ws_bytes(int B, int Hkv, const DecodeSplit& d) {
  const size_t parts = static_cast<size_t>(B) * Hkv * d.nhb * d.splits;
  return 16 + parts * 16 * 2 * sizeof(float) + parts * 16 * 128 * sizeof(float);
}

int device_sms(int* nsm) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(nsm, cudaDevAttrMultiProcessorCount, dev);
  if (major != 10) return fail(SWA_E_UNSUPPORTED, "this library targets sm_100 (B200) devices");
  return SWA_OK;
}

}  // namespace

size_t swa_decode_workspace_bytes(int B, int Smax, int Hq, int Hkv) {
  if (B <= 0 || Smax <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0) return 0;
  int nsm = 0;
  if (device_sms(&nsm) != SWA_OK) return 0;
  return decode_ws_bytes(B, Hkv, decode_split(B, Smax, Hq, Hkv, nsm));
}

}  // extern "C"

namespace {

int decode_forward_impl(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                        const float* v_scale, bool fp8, const int32_t* seq_lens, const uint8_t* route, void* out,
                        float* lse, int B, int Smax, int Hq, int Hkv, int head_dim, int window, float scale_log2,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (head_dim != 128) return fail(SWA_E_UNSUPPORTED, "head_dim must be 128");
  if (B <= 0 || Smax <= 0 || Hq <= 0 || Hkv <= 0) return fail(SWA_E_INVALID, "empty or negative shape");
  if (Hq % Hkv != 0) return fail(SWA_E_INVALID, "query heads must be divisible by KV heads");
  if (window <= 0) return fail(SWA_E_INVALID, "window_size must be positive");
  if (!(scale_log2 > 0.0f)) return fail(SWA_E_INVALID, "softmax scale must be positive");
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || seq_lens == nullptr || route == nullptr ||
      out == nullptr || lse == nullptr || workspace == nullptr)
    return fail(SWA_E_INVALID, "null pointer");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out) || !aligned16(workspace))
    return fail(SWA_E_INVALID, "q/k/v/out/workspace must be 16-byte aligned");
  if (static_cast<int64_t>(B) * Smax * Hkv >= (int64_t(1) << 31))
    return fail(SWA_E_UNSUPPORTED, "KV cache too large for 32-bit row indices");
  if (fp8 && (k_scale == nullptr || v_scale == nullptr)) return fail(SWA_E_INVALID, "FP8 cache needs k/v scales");
  int nsm = 0;
  int rc = device_sms(&nsm);
  if (rc != SWA_OK) return rc;
  const DecodeSplit d = decode_split(B, Smax, Hq, Hkv, nsm);
  if (B > 65535) return fail(SWA_E_UNSUPPORTED, "decode grid: at most 65535 sequences");
  if (workspace_bytes < decode_ws_bytes(B, Hkv, d)) return fail(SWA_E_INVALID, "workspace too small");

  swa::DecodeParams p{};
  if (fp8) {
    // bytes: 128 per (key, KV head); one box = 64 keys x 128 bytes
    const uint64_t kd[4] = {128, static_cast<uint64_t>(Hkv), static_cast<uint64_t>(Smax), static_cast<uint64_t>(B)};
    const uint64_t ks[3] = {128, static_cast<uint64_t>(Hkv) * 128, static_cast<uint64_t>(Smax) * Hkv * 128};
    const uint32_t kb[4] = {128, 1, 64, 1};
    if (!swa::make_u8_map_sw128(&p.k_map, k_cache, 4, kd, ks, kb)) return fail(SWA_E_TMA, "k tensor map");
    if (!swa::make_u8_map_sw128(&p.v_map, v_cache, 4, kd, ks, kb)) return fail(SWA_E_TMA, "v tensor map");
  } else {
    const uint64_t kd[4] = {128, static_cast<uint64_t>(Hkv), static_cast<uint64_t>(Smax), static_cast<uint64_t>(B)};
    const uint64_t ks[3] = {256, static_cast<uint64_t>(Hkv) * 256, static_cast<uint64_t>(Smax) * Hkv * 256};
    const uint32_t kb[4] = {64, 1, 64, 1};
    if (!swa::make_bf16_map_sw128(&p.k_map, k_cache, 4, kd, ks, kb)) return fail(SWA_E_TMA, "k tensor map");
    if (!swa::make_bf16_map_sw128(&p.v_map, v_cache, 4, kd, ks, kb)) return fail(SWA_E_TMA, "v tensor map");
  }
  p.fp8 = fp8 ? 1 : 0;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  const size_t parts = static_cast<size_t>(B) * Hkv * d.nhb * d.splits;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.status = reinterpret_cast<int32_t*>(ws);
  p.part_ml = reinterpret_cast<float*>(ws + 16);
  p.part_o = reinterpret_cast<float*>(ws + 16 + parts * 16 * 2 * sizeof(float));
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.seq_lens = seq_lens;
  p.route = route;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.B = B;
  p.Smax = Smax;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.r = Hq / Hkv;
  p.nhb = d.nhb;
  p.splits = d.splits;
  p.split_keys = d.split_keys;
  p.window = window;
  p.scale_log2 = scale_log2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(p.status, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "status reset");
  e = swa::launch_decode(p, s);
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return SWA_OK;
}

}  // namespace

extern "C" {

int swa_decode_forward(const void* q, const void* k_cache, const void* v_cache, const int32_t* seq_lens,
                       const uint8_t* route, void* out, float* lse, int B, int Smax, int Hq, int Hkv,
                       int head_dim, int window, float scale_log2, void* workspace, size_t workspace_bytes,
                       void* stream) {
  return decode_forward_impl(q, k_cache, v_cache, nullptr, nullptr, false, seq_lens, route, out, lse, B, Smax, Hq,
                             Hkv, head_dim, window, scale_log2, workspace, workspace_bytes, stream);
}

int swa_decode_forward_fp8(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                           const float* v_scale, const int32_t* seq_lens, const uint8_t* route, void* out, float* lse,
                           int B, int Smax, int Hq, int Hkv, int head_dim, int window, float scale_log2,
                           void* workspace, size_t workspace_bytes, void* stream) {
  return decode_forward_impl(q, k_cache, v_cache, k_scale, v_scale, true, seq_lens, route, out, lse, B, Smax, Hq,
                             Hkv, head_dim, window, scale_log2, workspace, workspace_bytes, stream);
}

size_t swa_backward_workspace_bytes(int B, int Hq, int full_stride, int local_stride) {
  if (B <= 0 || Hq <= 0 || full_stride < 0 || local_stride < 0) return 0;
  return swa::backward_workspace_bytes(B, Hq, full_stride, local_stride);
}

int swa_prefill_backward(const void* q, const void* k, const void* v, const void* o, const float* lse,
                         const void* dout, const int32_t* full_idx, const int32_t* local_idx, int full_stride,
                         int local_stride, const int32_t* counts, const int32_t* full_starts,
                         const int32_t* local_starts, const int32_t* causal_ends, void* dq, void* dk, void* dv,
                         int B, int Sq, int Skv, int Hq, int Hkv, int head_dim, int window, float scale_log2,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (head_dim != 128) return fail(SWA_E_UNSUPPORTED, "head_dim must be 128");
  if (B <= 0 || Sq <= 0 || Skv <= 0 || Hq <= 0 || Hkv <= 0) return fail(SWA_E_INVALID, "empty or negative shape");
  if (Hq % Hkv != 0) return fail(SWA_E_INVALID, "query heads must be divisible by KV heads");
  if (window <= 0) return fail(SWA_E_INVALID, "window_size must be positive");
  if (!(scale_log2 > 0.0f)) return fail(SWA_E_INVALID, "softmax scale must be positive");
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr || lse == nullptr || dout == nullptr ||
      dq == nullptr || dk == nullptr || dv == nullptr || counts == nullptr || workspace == nullptr)
    return fail(SWA_E_INVALID, "null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(dout) || !aligned16(dq) ||
      !aligned16(dk) || !aligned16(dv))
    return fail(SWA_E_INVALID, "tensors must be 16-byte aligned");
  if (full_stride < 0 || local_stride < 0 || (full_stride > 0 && full_idx == nullptr) ||
      (local_stride > 0 && local_idx == nullptr))
    return fail(SWA_E_INVALID, "bad index lists");
  const bool has_meta = causal_ends != nullptr;
  if (has_meta && (full_starts == nullptr || local_starts == nullptr))
    return fail(SWA_E_INVALID, "metadata needs full_starts, local_starts and causal_ends");
  if (static_cast<int64_t>(B) * Sq * Hq >= (int64_t(1) << 31) || static_cast<int64_t>(B) * Skv * Hkv >= (int64_t(1) << 31))
    return fail(SWA_E_UNSUPPORTED, "tensor too large for 32-bit row indices");
  const int fs = full_idx ? full_stride : 0, ls = local_idx ? local_stride : 0;
  if (static_cast<int64_t>(B) * Hq * (static_cast<int64_t>(fs) + ls) >= (int64_t(1) << 31))
    return fail(SWA_E_UNSUPPORTED, "index lists too wide for 32-bit packed row indices");
  if (!aligned16(workspace) || workspace_bytes < swa::backward_workspace_bytes(B, Hq, fs, ls))
    return fail(SWA_E_INVALID, "workspace must be 16-byte aligned and hold swa_backward_workspace_bytes() bytes");
  int nsm = 0;
  int rc = device_sms(&nsm);
  if (rc != SWA_OK) return rc;
  swa::BwdParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.o = static_cast<const __nv_bfloat16*>(o);
  p.dout = static_cast<const __nv_bfloat16*>(dout);
  p.lse = lse;
  p.idx[0] = full_idx;
  p.idx[1] = local_idx;
  p.idx_stride[0] = full_idx ? full_stride : 0;
  p.idx_stride[1] = local_idx ? local_stride : 0;
  p.counts = counts;
  p.starts[0] = full_starts;
  p.starts[1] = local_starts;
  p.ends = causal_ends;
  p.dq = static_cast<__nv_bfloat16*>(dq);
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.B = B;
  p.Sq = Sq;
  p.Skv = Skv;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.r = Hq / Hkv;
  p.window = window;
  p.scale_log2 = scale_log2;
  p.scale = scale_log2 / 1.4426950408889634f;
  for (int br = 0; br < 2; ++br)
    p.nblk[br] = static_cast<int>((static_cast<int64_t>(p.idx_stride[br]) * p.r + 127) / 128);
  swa::bind_backward_workspace(p, workspace);
  const uint64_t kd[4] = {128, static_cast<uint64_t>(Hkv), static_cast<uint64_t>(Skv), static_cast<uint64_t>(B)};
  const uint64_t ks[3] = {256, static_cast<uint64_t>(Hkv) * 256, static_cast<uint64_t>(Skv) * Hkv * 256};
  const uint32_t kb[4] = {64, 1, 64, 1};
  if (!swa::make_bf16_map_sw128(&p.k_map, k, 4, kd, ks, kb)) return fail(SWA_E_TMA, "k tensor map");
  if (!swa::make_bf16_map_sw128(&p.v_map, v, 4, kd, ks, kb)) return fail(SWA_E_TMA, "v tensor map");
  const uint64_t prow = static_cast<uint64_t>(p.pk_rows > 0 ? p.pk_rows : 1);
  const uint64_t pd[2] = {128, prow};
  const uint64_t ps[1] = {256};
  const uint32_t pb[2] = {64, 64};
  if (!swa::make_bf16_map_sw128(&p.qp_map, p.qp, 2, pd, ps, pb)) return fail(SWA_E_TMA, "packed q tensor map");
  if (!swa::make_bf16_map_sw128(&p.dop_map, p.dop, 2, pd, ps, pb)) return fail(SWA_E_TMA, "packed dout tensor map");
  if (!swa::make_i32_map_2d(&p.rec_map, p.rec, 4, prow, 16, 4, 64)) return fail(SWA_E_TMA, "row record tensor map");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // rows that no list routes keep a zero gradient
  cudaError_t e = cudaMemsetAsync(dq, 0, static_cast<size_t>(B) * Sq * Hq * 128 * 2, s);
  if (e != cudaSuccess) return cuda_fail(e, "dq reset");
  e = cudaMemsetAsync(p.status, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "status reset");
  e = swa::launch_backward(p, nsm, s);
  if (e != cudaSuccess) return cuda_fail(e, "backward launch");
  return SWA_OK;
}

}  // extern "C"

namespace {

// Row-major output replicas of a prefill launch (null: none).
struct Replicas {
  int n;
  int hkv;
  const int32_t* unit_gid;
  void* const* out;
  float* const* lse;
};

int prefill_forward_impl(const void* q, const void* k, const void* v, const int32_t* full_idx,
                         const int32_t* local_idx, int full_stride, int local_stride, int full_cap, int local_cap,
                         const int32_t* counts, int counts_batch_major, int count_full, int count_local,
                         const int32_t* full_starts, const int32_t* local_starts, const int32_t* causal_ends,
                         const int32_t* bg_list, int n_bg, void* out, float* lse, int B, int Sq, int Skv, int Hq,
                         int Hkv, int head_dim, int window, float scale_log2, const int32_t* gate,
                         int32_t* workspace, size_t workspace_bytes, void* stream, const Replicas* rep,
                         int split_tiles = 0, void* scratch = nullptr, size_t scratch_bytes = 0) {
  if (head_dim != 128) return fail(SWA_E_UNSUPPORTED, "head_dim must be 128");
  if (B <= 0 || Sq <= 0 || Skv <= 0 || Hq <= 0 || Hkv <= 0) return fail(SWA_E_INVALID, "empty or negative shape");
  if (Hq % Hkv != 0) return fail(SWA_E_INVALID, "query heads must be divisible by KV heads");
  if (window <= 0) return fail(SWA_E_INVALID, "window_size must be positive");
  if (!(scale_log2 > 0.0f)) return fail(SWA_E_INVALID, "softmax scale must be positive");
  const bool replicated = rep != nullptr && rep->n > 0;
  if (q == nullptr || k == nullptr || v == nullptr || ((out == nullptr || lse == nullptr) && !replicated))
    return fail(SWA_E_INVALID, "null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (out != nullptr && !aligned16(out)))
    return fail(SWA_E_INVALID, "q/k/v/out must be 16-byte aligned");
  if ((out == nullptr) != (lse == nullptr)) return fail(SWA_E_INVALID, "out and lse are both given or both null");
  if (replicated) {
    if (rep->n > swa::kMaxReplicas) return fail(SWA_E_INVALID, "at most 8 replicas");
    if (Hkv != 1) return fail(SWA_E_INVALID, "replicated outputs need a unit-major launch (Hkv == 1)");
    if (rep->hkv <= 0 || rep->unit_gid == nullptr || rep->out == nullptr || rep->lse == nullptr)
      return fail(SWA_E_INVALID, "replicas need unit ids, the global KV head count and output pointers");
    for (int t = 0; t < rep->n; ++t)
      if (rep->out[t] == nullptr || rep->lse[t] == nullptr || !aligned16(rep->out[t]))
        return fail(SWA_E_INVALID, "replica outputs must be non-null and 16-byte aligned");
    if (static_cast<int64_t>(B) * Sq * Hq >= (int64_t(1) << 31))
      return fail(SWA_E_UNSUPPORTED, "tensor too large for 32-bit row indices");
  }
  if (workspace == nullptr || workspace_bytes < 16) return fail(SWA_E_INVALID, "workspace must hold 16 bytes");
  if (counts == nullptr && B != 1) return fail(SWA_E_INVALID, "device counts are required when B > 1");
  if (full_cap < 0 || local_cap < 0 || (full_cap > 0 && full_idx == nullptr) ||
      (local_cap > 0 && local_idx == nullptr))
    return fail(SWA_E_INVALID, "bad index lists");
  if (full_cap > full_stride && B > 1) return fail(SWA_E_INVALID, "full_cap exceeds full_stride");
  if (local_cap > local_stride && B > 1) return fail(SWA_E_INVALID, "local_cap exceeds local_stride");
  const bool has_meta = causal_ends != nullptr;
  if (has_meta && (full_starts == nullptr || local_starts == nullptr))
    return fail(SWA_E_INVALID, "metadata needs full_starts, local_starts and causal_ends");
  if (bg_list != nullptr && n_bg <= 0) return fail(SWA_E_INVALID, "empty unit list");
  if (static_cast<int64_t>(B) * Sq * Hq >= (int64_t(1) << 31) || static_cast<int64_t>(B) * Skv * Hkv >= (int64_t(1) << 31))
    return fail(SWA_E_UNSUPPORTED, "tensor too large for 32-bit row indices");

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int major = 0, nsm = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (major != 10) return fail(SWA_E_UNSUPPORTED, "this library targets sm_100 (B200) devices");

  const int r = Hq / Hkv;
  int rp = r & (-r);  // largest power of two dividing the group size
  if (rp > 256) rp = 256;

  swa::PrefillParams p{};
  {
    const uint64_t qd[2] = {128, static_cast<uint64_t>(B) * Sq * Hq};
    const uint64_t qs[1] = {256};
    const uint32_t qb[2] = {64, static_cast<uint32_t>(rp < 128 ? rp : 128)};
    if (!swa::make_bf16_map_sw128(&p.q_map, q, 2, qd, qs, qb)) return fail(SWA_E_TMA, "q tensor map");
    // runs of consecutive routed positions: one box covers 2^(L+1) positions x rp heads
    p.n_q3 = 0;
    if (rp <= 64) {
      const uint64_t q3d[3] = {128, static_cast<uint64_t>(Hq), static_cast<uint64_t>(B) * Sq};
      const uint64_t q3s[2] = {256, static_cast<uint64_t>(Hq) * 256};
      for (int npos = 2; npos * rp <= 128 && p.n_q3 < swa::kMaxQRunMaps; npos *= 2) {
        const uint32_t q3b[3] = {64, static_cast<uint32_t>(rp), static_cast<uint32_t>(npos)};
        if (!swa::make_bf16_map_sw128(&p.q_runs[p.n_q3], q, 3, q3d, q3s, q3b)) return fail(SWA_E_TMA, "q run tensor map");
        ++p.n_q3;
      }
    }
    // one box per 128-key K or V tile: dims (64 columns, key, column half, KV head,
    // batch), box {64, 128, 2, 1, 1}, so the tile lands as its two 64-column halves
    // of 128 swizzled rows each (16 KB apart), in one TMA instruction
    const uint64_t kd[5] = {64, static_cast<uint64_t>(Skv), 2, static_cast<uint64_t>(Hkv), static_cast<uint64_t>(B)};
    const uint64_t ks[4] = {static_cast<uint64_t>(Hkv) * 256, 128, 256, static_cast<uint64_t>(Skv) * Hkv * 256};
    const uint32_t kb[5] = {64, 128, 2, 1, 1};
    if (!swa::make_bf16_map_sw128(&p.k_map, k, 5, kd, ks, kb)) return fail(SWA_E_TMA, "k tensor map");
    if (!swa::make_bf16_map_sw128(&p.v_map, v, 5, kd, ks, kb)) return fail(SWA_E_TMA, "v tensor map");
  }
  p.idx[0] = full_idx;
  p.idx[1] = local_idx;
  p.idx_stride[0] = full_stride;
  p.idx_stride[1] = local_stride;
  p.idx_cap[0] = full_idx ? full_cap : 0;
  p.idx_cap[1] = local_idx ? local_cap : 0;
  p.counts = counts;
  p.cs_branch = counts_batch_major ? 1 : B;
  p.cs_batch = counts_batch_major ? 2 : 1;
  p.count_scalar[0] = count_full;
  p.count_scalar[1] = count_local;
  p.starts[0] = full_starts;
  p.starts[1] = local_starts;
  p.ends = causal_ends;
  p.bg_list = bg_list;
  p.n_bg = bg_list ? n_bg : B * Hkv;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.counter = workspace;
  p.status = workspace + 1;
  p.gate = gate;
  p.B = B;
  p.Sq = Sq;
  p.Skv = Skv;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.window = window;
  p.scale_log2 = scale_log2;
  p.rp = rp;
  p.pc = 256 / rp;
  p.nhb = r / rp;
  p.boxh = rp < 128 ? rp : 128;
  p.test_withhold = g_test_withhold.load();
  if (replicated) {
    p.n_rep = rep->n;
    p.rep_hkv = rep->hkv;
    p.unit_gid = rep->unit_gid;
    for (int t = 0; t < rep->n; ++t) {
      p.rep_out[t] = static_cast<__nv_bfloat16*>(rep->out[t]);
      p.rep_lse[t] = rep->lse[t];
    }
  }

  p.pieces = 1;
  const int64_t n_max_tiles = (static_cast<int64_t>(Skv) + 127) / 128;
  if (split_tiles > 0 && p.idx_cap[0] > 0 && n_max_tiles > split_tiles) {
    // pieces per full-branch unit from the piece length; scratch slots for the
    // longest units of every (unit, head block), as many as the scratch holds (the
    // plan's bytes give one per position block the counts allow; units ranked
    // beyond the scratch run whole)
    if (replicated) return fail(SWA_E_INVALID, "a key split cannot be combined with replicated outputs");
    const int64_t pieces = (n_max_tiles + split_tiles - 1) / split_tiles;
    const int64_t pb_cap = (static_cast<int64_t>(p.idx_cap[0]) + p.pc - 1) / p.pc;
    const int64_t per_rank = static_cast<int64_t>(p.nhb) * p.n_bg * pieces * swa::kSplitSlotBytes;
    const int64_t k_cap = std::min<int64_t>(pb_cap, static_cast<int64_t>(scratch_bytes) / per_rank);
    if (scratch == nullptr || !aligned16(scratch) || k_cap < 1)
      return fail(SWA_E_INVALID, "key-split scratch missing, unaligned or smaller than one slot per unit");
    const int64_t slots = k_cap * p.nhb * p.n_bg * pieces;
    p.pieces = static_cast<int>(pieces);
    p.split_tiles = split_tiles;
    p.split_pb_cap = static_cast<int>(k_cap);
    p.part_lse = static_cast<float*>(scratch);
    p.part_o = static_cast<float*>(scratch) + slots * 256;
  }

  const int64_t per_level = static_cast<int64_t>(p.n_bg) * p.nhb;
  const int64_t items = (static_cast<int64_t>(p.idx_cap[0] + p.pc - 1) / p.pc * p.pieces +
                         (p.idx_cap[1] + p.pc - 1) / p.pc) * per_level;
  if (items == 0) return SWA_OK;
  if (items >= (int64_t(1) << 31)) return fail(SWA_E_UNSUPPORTED, "too many work items");
  const int ctas = static_cast<int>(items < nsm ? items : nsm);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(workspace, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "workspace reset");
  e = swa::launch_prefill(p, ctas, s);
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  e = swa::launch_merge_pieces(p, s);
  if (e != cudaSuccess) return cuda_fail(e, "key-split merge launch");
  return SWA_OK;
}

}  // namespace

extern "C" {

int swa_prefill_forward(const void* q, const void* k, const void* v, const int32_t* full_idx,
                        const int32_t* local_idx, int full_stride, int local_stride, int full_cap, int local_cap,
                        const int32_t* counts, int counts_batch_major, int count_full, int count_local,
                        const int32_t* full_starts,
                        const int32_t* local_starts, const int32_t* causal_ends, const int32_t* bg_list, int n_bg,
                        void* out, float* lse, int B, int Sq, int Skv, int Hq, int Hkv, int head_dim, int window,
                        float scale_log2, const int32_t* gate, int32_t* workspace, size_t workspace_bytes,
                        void* stream) {
  return prefill_forward_impl(q, k, v, full_idx, local_idx, full_stride, local_stride, full_cap, local_cap, counts,
                              counts_batch_major, count_full, count_local, full_starts, local_starts, causal_ends,
                              bg_list, n_bg, out, lse, B, Sq, Skv, Hq, Hkv, head_dim, window, scale_log2, gate,
                              workspace, workspace_bytes, stream, nullptr);
}

size_t swa_prefill_split_plan(int B, int Skv, int Hq, int Hkv, int full_cap, int local_cap, int n_bg, int window,
                              int num_sms, int request_tiles, int* split_tiles) {
  if (split_tiles != nullptr) *split_tiles = 0;
  if (B <= 0 || Skv <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || full_cap < 0 || local_cap < 0 || window <= 0)
    return 0;
  const int r = Hq / Hkv;
  int rp = r & (-r);
  if (rp > 256) rp = 256;
  const int n_units = n_bg > 0 ? n_bg : B * Hkv;
  const swa::SplitPlan plan =
      swa::plan_split(n_units, r / rp, 256 / rp, full_cap, local_cap, Skv, window, num_sms, request_tiles);
  if (split_tiles != nullptr) *split_tiles = plan.tiles;
  return plan.tiles > 0 ? plan.bytes : 0;
}

int swa_prefill_forward_split(const void* q, const void* k, const void* v, const int32_t* full_idx,
                              const int32_t* local_idx, int full_stride, int local_stride, int full_cap, int local_cap,
                              const int32_t* counts, int counts_batch_major, int count_full, int count_local,
                              const int32_t* full_starts, const int32_t* local_starts, const int32_t* causal_ends,
                              const int32_t* bg_list, int n_bg, void* out, float* lse, int B, int Sq, int Skv, int Hq,
                              int Hkv, int head_dim, int window, float scale_log2, const int32_t* gate,
                              int32_t* workspace, size_t workspace_bytes, int split_tiles, void* scratch,
                              size_t scratch_bytes, void* stream) {
  if (split_tiles < 0) return fail(SWA_E_INVALID, "split_tiles must be non-negative");
  return prefill_forward_impl(q, k, v, full_idx, local_idx, full_stride, local_stride, full_cap, local_cap, counts,
                              counts_batch_major, count_full, count_local, full_starts, local_starts, causal_ends,
                              bg_list, n_bg, out, lse, B, Sq, Skv, Hq, Hkv, head_dim, window, scale_log2, gate,
                              workspace, workspace_bytes, stream, nullptr, split_tiles, scratch, scratch_bytes);
}

int swa_prefill_forward_replicated(const void* q, const void* k, const void* v, const int32_t* full_idx,
                                   const int32_t* local_idx, int full_stride, int local_stride,
                                   const int32_t* counts, const int32_t* full_starts, const int32_t* local_starts,
                                   const int32_t* causal_ends, const int32_t* unit_gid, int B, int Sq, int Skv, int Hq,
                                   int head_dim, int window, float scale_log2, int rep_hkv, int n_rep,
                                   void* const* rep_out, float* const* rep_lse, void* out, float* lse,
                                   int32_t* workspace, size_t workspace_bytes, void* stream) {
  if (n_rep <= 0) return fail(SWA_E_INVALID, "n_rep must be at least 1");
  const Replicas rep{n_rep, rep_hkv, unit_gid, rep_out, rep_lse};
  return prefill_forward_impl(q, k, v, full_idx, local_idx, full_stride, local_stride, full_stride, local_stride,
                              counts, 1, 0, 0, full_starts, local_starts, causal_ends, nullptr, 0, out, lse, B, Sq,
                              Skv, Hq, 1, head_dim, window, scale_log2, nullptr, workspace, workspace_bytes, stream,
                              &rep);
}

}  // extern "C"
