// Routing-mask compaction, capacity-bucket preparation / validation and varlen
// metadata for the Switch Attention prefill path (sm_100a).
//
// These kernels are HBM/latency-bound integer work: coalesced 16-byte loads,
// warp ballots and block scans, no tensor cores.
#include "swattn_internal.h"

namespace swa {

namespace {

constexpr int kCompactThreads = 1024;
constexpr int kCompactPerThread = 16;

__device__ __forceinline__ int warp_inclusive_scan(int v) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) >= o) v += n;
  }
  return v;
}

// Routing decisions of 16 consecutive tokens as a bit mask (bit i = token e0 + i
// goes to full attention), read from a uint8 / bool mask (non-zero = full).
struct MaskReader {
  const uint8_t* m;  // this batch row
  __device__ __forceinline__ uint32_t bits(int e0, int nvalid, bool vec_ok) const {
    uint32_t bits = 0;
    if (nvalid == 16 && vec_ok) {
      const uint4 w = *reinterpret_cast<const uint4*>(m + e0);
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int by = 0; by < 4; ++by)
          if ((words[q] >> (8 * by)) & 0xFFu) bits |= 1u << (q * 4 + by);
    } else {
      for (int i = 0; i < nvalid; ++i)
        if (m[e0 + i]) bits |= 1u << i;
    }
    return bits;
  }
};

__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

// Routing decisions from router outputs of type T (BF16 or FP32), compared in
// FP32: kPair = 0, one score per token, full iff score > threshold; kPair = 1,
// two logits per token (local, full), full iff logit_full - logit_local >
// threshold (threshold 0 = argmax, ties to local).  NaN routes to local.
template <typename T, int kPair>
struct RouterReader {
  const T* r;  // this batch row: S * (1 + kPair) values
  float threshold;
  __device__ __forceinline__ bool full_at(const T* v) const {
    if (kPair) return to_float(v[1]) - to_float(v[0]) > threshold;
    return to_float(v[0]) > threshold;
  }
  __device__ __forceinline__ uint32_t bits(int e0, int nvalid, bool vec_ok) const {
    constexpr int kPer = 1 + kPair;
    constexpr int kVec = 16 * kPer * static_cast<int>(sizeof(T)) / 16;  // uint4 loads per 16 tokens
    uint32_t bits = 0;
    const T* base = r + static_cast<int64_t>(e0) * kPer;
    if (nvalid == 16 && vec_ok) {
      uint4 w[kVec];
#pragma unroll
      for (int i = 0; i < kVec; ++i) w[i] = reinterpret_cast<const uint4*>(base)[i];
      const T* v = reinterpret_cast<const T*>(w);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (full_at(v + kPer * i)) bits |= 1u << i;
    } else {
      for (int i = 0; i < nvalid; ++i)
        if (full_at(base + kPer * i)) bits |= 1u << i;
    }
    return bits;
  }
};

// One CTA per batch row.  Each pass covers 16384 tokens: every thread turns the
// routing decisions of its 16 tokens into a bit mask, a block-wide exclusive
// scan of the popcounts gives each thread its first slot in the full list (the
// local slot follows from the token index), and the positions are written in
// increasing order.  For a mask the result equals positions[mask] /
// positions[~mask] (reference swiattn_gqa_prefill_varlen.py:321-322) bit for
// bit; the tails of both [B, S] buffers are filled with -1.
template <typename Reader>
__device__ __forceinline__ void compact_row(const Reader& rd, bool vec_ok, int S, int b, int32_t* __restrict__ full,
                                            int32_t* __restrict__ local, int32_t* __restrict__ counts) {
  int32_t* f = full + static_cast<int64_t>(b) * S;
  int32_t* l = local + static_cast<int64_t>(b) * S;
  __shared__ int warp_sums[32];
  __shared__ int chunk_total;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int base_full = 0;
  for (int c0 = 0; c0 < S; c0 += kCompactThreads * kCompactPerThread) {
    const int e0 = c0 + threadIdx.x * kCompactPerThread;
    const int nvalid = max(0, min(kCompactPerThread, S - e0));
    const uint32_t bits = nvalid > 0 ? rd.bits(e0, nvalid, vec_ok) : 0u;
    const int cf = __popc(bits);
    const int incl = warp_inclusive_scan(cf);
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int v = warp_sums[lane];
      const int vi = warp_inclusive_scan(v);
      warp_sums[lane] = vi - v;
      if (lane == 31) chunk_total = vi;
    }
    __syncthreads();
    int fi = base_full + warp_sums[warp] + incl - cf;  // full slot of this thread's first full element
    int li = e0 - fi;                                   // local slot of its first local element
    for (int i = 0; i < nvalid; ++i) {
      if ((bits >> i) & 1u)
        f[fi++] = e0 + i;
      else
        l[li++] = e0 + i;
    }
    base_full += chunk_total;
    __syncthreads();
  }
  const int n_full = base_full;
  const int n_local = S - base_full;
  if (threadIdx.x == 0) {
    counts[2 * b] = n_full;
    counts[2 * b + 1] = n_local;
  }
  for (int i = threadIdx.x; i < S; i += kCompactThreads) {
    if (i >= n_full) f[i] = -1;
    if (i >= n_local) l[i] = -1;
  }
}

__global__ void __launch_bounds__(kCompactThreads) compact_mask_kernel(const uint8_t* __restrict__ mask, int S,
                                                                        int32_t* __restrict__ full,
                                                                        int32_t* __restrict__ local,
                                                                        int32_t* __restrict__ counts) {
  const MaskReader rd{mask + static_cast<int64_t>(blockIdx.x) * S};
  compact_row(rd, (reinterpret_cast<uintptr_t>(rd.m) & 15u) == 0, S, blockIdx.x, full, local, counts);
}

// Router outputs -> routing decision -> compaction in one pass (no mask buffer).
template <typename T, int kPair>
__global__ void __launch_bounds__(kCompactThreads) compact_router_kernel(const T* __restrict__ router,
                                                                          float threshold, int S,
                                                                          int32_t* __restrict__ full,
                                                                          int32_t* __restrict__ local,
                                                                          int32_t* __restrict__ counts) {
  const RouterReader<T, kPair> rd{router + static_cast<int64_t>(blockIdx.x) * S * (1 + kPair), threshold};
  compact_row(rd, (reinterpret_cast<uintptr_t>(rd.r) & 15u) == 0, S, blockIdx.x, full, local, counts);
}

// Capacity-bucket preparation of one index list per batch row (reference
// _prepare_indices, swiattn_gqa_prefill_varlen.py:271-304): copy to the padded
// [B, cap] buffer with -1 fill, count the valid entries and record range /
// strict-increase violations in the status word.  pad_bit == 0 selects the
// reference's exact-length form (all N entries valid); otherwise -1 entries are
// trailing padding and a valid entry after padding sets pad_bit.
__global__ void prepare_indices_kernel(const int32_t* __restrict__ idx, int N, int seq_len, int cap,
                                       int32_t* __restrict__ padded, int32_t* __restrict__ count,
                                       int32_t* __restrict__ status, int range_bit, int order_bit, int pad_bit) {
  const int b = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int32_t* row = idx + static_cast<int64_t>(b) * N;
  int flags = 0;
  int valid_here = 0;
  int v = -1;
  if (i < N) {
    v = row[i];
    if (pad_bit == 0 || v != -1) {
      valid_here = 1;
      if (v < 0 || v >= seq_len) flags |= range_bit;
      if (i > 0) {
        const int pv = row[i - 1];
        if (pad_bit != 0 && pv == -1)
          flags |= pad_bit;
        else if (v <= pv)
          flags |= order_bit;
      }
    }
  }
  if (padded != nullptr && i < cap) padded[static_cast<int64_t>(b) * cap + i] = i < N ? v : -1;
  const unsigned ballot = __ballot_sync(0xffffffffu, valid_here);
  int f = flags;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) f |= __shfl_xor_sync(0xffffffffu, f, o);
  if ((threadIdx.x & 31) == 0) {
    if (pad_bit != 0 && ballot) atomicAdd(count + b, __popc(ballot));
    if (f) atomicOr(status, f);
  }
  if (pad_bit == 0 && i == 0) count[b] = N;
}

__global__ void check_cover_kernel(const int32_t* __restrict__ counts, int B, int seq_len, int32_t* status) {
  for (int b = threadIdx.x; b < B; b += blockDim.x)
    if (counts[b] + counts[B + b] != seq_len) atomicOr(status, kStatusCover);
}

// Varlen metadata (the reference's missing metadata module, semantics inferred
// from swiattn_gqa_prefill_varlen.py:134-137,186-196): for row t of segment s,
// full_starts = cu[s], local_starts = max(cu[s], t - W + 1), causal_ends = t + 1,
// q_positions = t - cu[s], segment ids = s.  Without cu_seqlens the whole
// sequence is one segment and the kv vectors are arange(kv_len) / zeros.
__global__ void build_metadata_kernel(const int32_t* __restrict__ cu, int nseg, int q_len, int kv_len, int window,
                                      int32_t* q_positions, int32_t* kv_positions, int32_t* q_segment_ids,
                                      int32_t* kv_segment_ids, int32_t* full_starts, int32_t* local_starts,
                                      int32_t* causal_ends) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t < q_len) {
    int seg = 0, start = 0;
    if (cu != nullptr) {
      int lo = 0, hi = nseg - 1;  // largest s with cu[s] <= t
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (cu[mid] <= t)
          lo = mid;
        else
          hi = mid - 1;
      }
      seg = lo;
      start = cu[lo];
    }
    q_positions[t] = t - start;
    q_segment_ids[t] = seg;
    full_starts[t] = start;
    local_starts[t] = max(start, t - window + 1);
    causal_ends[t] = t + 1;
    if (cu != nullptr && t < kv_len) {
      kv_positions[t] = t - start;
      kv_segment_ids[t] = seg;
    }
  }
  if (cu == nullptr && t < kv_len) {
    kv_positions[t] = t;
    kv_segment_ids[t] = 0;
  }
}


// Multi-CTA compaction of long rows: chunks of kChunk tokens, one CTA of
// kChunkThreads threads (16 tokens each) per (chunk, row), in two launches.
// Pass 1 stores each chunk's number of full tokens in the workspace.  Pass 2
// sums the counts of the row's earlier chunks (its first full slot), runs the
// same block scan as compact_row over its chunk and writes the positions; it
// also writes -1 to the list slots of its own index range that lie past the
// row's counts, so every output slot has exactly one writer.  Rows of at most
// one chunk take the single-CTA kernels above.
constexpr int kChunkThreads = 256;
constexpr int kChunk = kChunkThreads * kCompactPerThread;  // 4096 tokens

struct MaskSource {
  const uint8_t* mask;
  int S;
  __device__ __forceinline__ MaskReader row(int b) const { return MaskReader{mask + static_cast<int64_t>(b) * S}; }
  __device__ __forceinline__ bool aligned(int b) const {
    return (reinterpret_cast<uintptr_t>(mask + static_cast<int64_t>(b) * S) & 15u) == 0;
  }
};

template <typename T, int kPair>
struct RouterSource {
  const T* router;
  float threshold;
  int S;
  __device__ __forceinline__ RouterReader<T, kPair> row(int b) const {
    return RouterReader<T, kPair>{router + static_cast<int64_t>(b) * S * (1 + kPair), threshold};
  }
  __device__ __forceinline__ bool aligned(int b) const {
    return (reinterpret_cast<uintptr_t>(router + static_cast<int64_t>(b) * S * (1 + kPair)) & 15u) == 0;
  }
};

__device__ __forceinline__ int block_sum_256(int v, int* red) {
  v = __reduce_add_sync(0xffffffffu, v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int w = 0; w < kChunkThreads / 32; ++w) t += red[w];
  __syncthreads();
  return t;
}

template <typename Source>
__global__ void __launch_bounds__(kChunkThreads) count_chunks_kernel(Source src, int S, int nch,
                                                                     int32_t* __restrict__ chunk_full) {
  __shared__ int red[kChunkThreads / 32];
  const int c = blockIdx.x, b = blockIdx.y;
  const int e0 = c * kChunk + threadIdx.x * kCompactPerThread;
  const int nvalid = max(0, min(kCompactPerThread, S - e0));
  const uint32_t bits = nvalid > 0 ? src.row(b).bits(e0, nvalid, src.aligned(b)) : 0u;
  const int total = block_sum_256(__popc(bits), red);
  if (threadIdx.x == 0) chunk_full[static_cast<int64_t>(b) * nch + c] = total;
}

template <typename Source>
__global__ void __launch_bounds__(kChunkThreads) write_chunks_kernel(Source src, int S, int nch,
                                                                     const int32_t* __restrict__ chunk_full,
                                                                     int32_t* __restrict__ full,
                                                                     int32_t* __restrict__ local,
                                                                     int32_t* __restrict__ counts) {
  __shared__ int red[kChunkThreads / 32];
  __shared__ int warp_sums[kChunkThreads / 32];
  const int c = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t* cf_row = chunk_full + static_cast<int64_t>(b) * nch;
  // full tokens before this chunk, and in the whole row
  int before = 0, all = 0;
  for (int i = threadIdx.x; i < nch; i += kChunkThreads) {
    const int v = cf_row[i];
    all += v;
    if (i < c) before += v;
  }
  before = block_sum_256(before, red);
  all = block_sum_256(all, red);
  const int e0 = c * kChunk + threadIdx.x * kCompactPerThread;
  const int nvalid = max(0, min(kCompactPerThread, S - e0));
  const uint32_t bits = nvalid > 0 ? src.row(b).bits(e0, nvalid, src.aligned(b)) : 0u;
  const int cf = __popc(bits);
  const int incl = warp_inclusive_scan(cf);
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int v = lane < kChunkThreads / 32 ? warp_sums[lane] : 0;
    const int vi = warp_inclusive_scan(v);
    if (lane < kChunkThreads / 32) warp_sums[lane] = vi - v;
  }
  __syncthreads();
  int32_t* f = full + static_cast<int64_t>(b) * S;
  int32_t* l = local + static_cast<int64_t>(b) * S;
  int fi = before + warp_sums[warp] + incl - cf;
  int li = e0 - fi;
  for (int i = 0; i < nvalid; ++i) {
    if ((bits >> i) & 1u)
      f[fi++] = e0 + i;
    else
      l[li++] = e0 + i;
  }
  const int n_full = all, n_local = S - all;
  const int i0 = c * kChunk, i1 = min(S, i0 + kChunk);
  for (int i = i0 + threadIdx.x; i < i1; i += kChunkThreads) {
    if (i >= n_full) f[i] = -1;
    if (i >= n_local) l[i] = -1;
  }
  if (c == 0 && threadIdx.x == 0) {
    counts[2 * b] = n_full;
    counts[2 * b + 1] = n_local;
  }
}

template <typename Source>
cudaError_t launch_chunked(const Source& src, int B, int S, int32_t* ws, int32_t* full, int32_t* local,
                           int32_t* counts, cudaStream_t stream) {
  const int nch = (S + kChunk - 1) / kChunk;
  const dim3 grid(nch, B);
  count_chunks_kernel<Source><<<grid, kChunkThreads, 0, stream>>>(src, S, nch, ws);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  write_chunks_kernel<Source><<<grid, kChunkThreads, 0, stream>>>(src, S, nch, ws, full, local, counts);
  return cudaGetLastError();
}

}  // namespace

int64_t compact_workspace_elems(int B, int S) {
  if (B <= 0 || S <= kChunk) return 0;
  return static_cast<int64_t>(B) * ((S + kChunk - 1) / kChunk);
}

cudaError_t launch_compact_mask(const uint8_t* mask, int B, int S, int32_t* full, int32_t* local, int32_t* counts,
                                int32_t* ws, cudaStream_t stream) {
  if (B <= 0) return cudaSuccess;
  if (ws != nullptr && S > kChunk) return launch_chunked(MaskSource{mask, S}, B, S, ws, full, local, counts, stream);
  compact_mask_kernel<<<B, kCompactThreads, 0, stream>>>(mask, S, full, local, counts);
  return cudaGetLastError();
}

cudaError_t launch_compact_router(const void* router, int dtype, int pair, float threshold, int B, int S,
                                  int32_t* full, int32_t* local, int32_t* counts, int32_t* ws, cudaStream_t stream) {
  if (B <= 0) return cudaSuccess;
  const bool chunked = ws != nullptr && S > kChunk;
  const dim3 grid(B);
  if (dtype == kRouterBf16) {
    const auto* r = static_cast<const __nv_bfloat16*>(router);
    if (pair) {
      if (chunked) return launch_chunked(RouterSource<__nv_bfloat16, 1>{r, threshold, S}, B, S, ws, full, local, counts, stream);
      compact_router_kernel<__nv_bfloat16, 1><<<grid, kCompactThreads, 0, stream>>>(r, threshold, S, full, local, counts);
    } else {
      if (chunked) return launch_chunked(RouterSource<__nv_bfloat16, 0>{r, threshold, S}, B, S, ws, full, local, counts, stream);
      compact_router_kernel<__nv_bfloat16, 0><<<grid, kCompactThreads, 0, stream>>>(r, threshold, S, full, local, counts);
    }
  } else {
    const auto* r = static_cast<const float*>(router);
    if (pair) {
      if (chunked) return launch_chunked(RouterSource<float, 1>{r, threshold, S}, B, S, ws, full, local, counts, stream);
      compact_router_kernel<float, 1><<<grid, kCompactThreads, 0, stream>>>(r, threshold, S, full, local, counts);
    } else {
      if (chunked) return launch_chunked(RouterSource<float, 0>{r, threshold, S}, B, S, ws, full, local, counts, stream);
      compact_router_kernel<float, 0><<<grid, kCompactThreads, 0, stream>>>(r, threshold, S, full, local, counts);
    }
  }
  return cudaGetLastError();
}

cudaError_t launch_prepare_indices(const int32_t* idx, int B, int N, int seq_len, int padded_rows, int cap,
                                   int32_t* padded, int32_t* count, int32_t* status, int range_bit, int order_bit,
                                   int pad_bit, cudaStream_t stream) {
  (void)padded_rows;
  if (B <= 0) return cudaSuccess;
  if (pad_bit != 0) {
    cudaError_t e = cudaMemsetAsync(count, 0, sizeof(int32_t) * B, stream);
    if (e != cudaSuccess) return e;
  }
  const int span = max(max(N, cap), 1);
  dim3 grid((span + 255) / 256, B);
  prepare_indices_kernel<<<grid, 256, 0, stream>>>(idx, N, seq_len, cap, padded, count, status, range_bit, order_bit,
                                                   pad_bit);
  return cudaGetLastError();
}

cudaError_t launch_check_cover(const int32_t* counts, int B, int seq_len, int32_t* status, cudaStream_t stream) {
  check_cover_kernel<<<1, 256, 0, stream>>>(counts, B, seq_len, status);
  return cudaGetLastError();
}

cudaError_t launch_build_metadata(const int32_t* cu_seqlens, int nseg, int q_len, int kv_len, int window,
                                  int32_t* q_positions, int32_t* kv_positions, int32_t* q_segment_ids,
                                  int32_t* kv_segment_ids, int32_t* full_starts, int32_t* local_starts,
                                  int32_t* causal_ends, cudaStream_t stream) {
  const int n = max(max(q_len, kv_len), 1);
  build_metadata_kernel<<<(n + 255) / 256, 256, 0, stream>>>(cu_seqlens, nseg, q_len, kv_len, window, q_positions,
                                                             kv_positions, q_segment_ids, kv_segment_ids,
                                                             full_starts, local_starts, causal_ends);
  return cudaGetLastError();
}

}  // namespace swa
