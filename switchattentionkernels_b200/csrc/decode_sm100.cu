// Switch Attention GQA decode step on B200 (sm_100a): one new query token per
// sequence attends to its KV cache, through full causal attention (keys
// [0, L)) or the causal sliding window (keys [max(0, L - W), L)), where L is
// the sequence's cached length including the new token.  This is the
// reference's row semantics (swiattn_gqa_prefill.py:145-158) at the last
// position t = L - 1 of each sequence, with the routing decided per sequence.
//
// The step is HBM-bound: every K/V element is read once and used by the r
// query heads of its group (about r FLOP per byte).  Layout of the work:
//   grid (split, KV group x head block, batch); a head block is 16 query heads
//   of one group (rows beyond r are zero), a split a contiguous range of the
//   sequence's legal keys.
//   warp 4  producer : TMA loads of 64-key K and V tiles (128B swizzle, two
//                      64-dim halves each) into a 2-entry ring (mbarriers).
//   warps 0-3 math   : warp w takes keys [16 w, 16 w + 16) of every tile:
//                      S = Q K^T and O += P V with mma.sync m16n8k16 (BF16 in,
//                      FP32 accumulate; the 16-row M dimension holds the
//                      head block), online softmax in the log2 domain (the
//                      running max raised, and O rescaled, only when it grows
//                      by more than 8), P rounded to BF16 before P V as in the
//                      prefill path.
//   FP8 e4m3 cache (switch_decode_kernel<true>): 64-key K and V byte tiles in a
//   4-entry ring; the math warps load their fragments from the bytes and
//   convert them to FP16 in registers (FP16 products, k_scale folded into the
//   score scale, v_scale into the merge).
//   The four warps' (max, sum, O) are merged in shared memory; the split's
//   partial goes to the workspace and a second kernel merges the splits and
//   writes O (BF16) and LSE (FP32, log2 units).
// Tensor cores run far below their peak here (M = 16 covers r <= 16 heads);
// the bound is HBM bandwidth.  Three CTAs per SM (2-entry rings, 69 KB of
// shared memory each) keep the loads in flight and give every scheduler three
// math warps to hide the mma.sync / ldmatrix latencies; one CTA per SM with a
// 4-entry ring streamed 15 % slower on the mixed batch and 26 % slower on
// all-window batches.
#include "mma_sync.cuh"
#include "sm100.cuh"
#include "swattn_internal.h"

namespace swa {

namespace {

constexpr int kDecStages = 2;
constexpr int kDecTileKeys = 64;
constexpr int kDecHalfBytes = kDecTileKeys * 128;        // 64 keys x 64 dims x 2 B
constexpr int kDecStageBytes = 4 * kDecHalfBytes;        // K h0, K h1, V h0, V h1
// FP8 cache: a stage is the K and V tiles as bytes (64 keys x 128 B each, 128B
// swizzle), 16 KB; four of them fill the 64 KB of the two BF16 stages.  The math
// warps read their MMA fragments straight from the byte tiles (ldmatrix on the
// bytes as 16-bit elements) and convert them in registers.
constexpr int kDecStageBytes8 = 2 * kDecTileKeys * 128;
constexpr float kDecRescale = 8.0f;  // log2 units: running-max growth that forces an O rescale
constexpr int kDecStages8 = 4;
constexpr int kDecMaxStages = 4;
static_assert(kDecStages8 * kDecStageBytes8 <= kDecStages * kDecStageBytes, "FP8 stages in the BF16 stage region");
constexpr int kDecThreads = 160;                         // 4 math warps + 1 producer warp
constexpr int kDecQBytes = 2 * 16 * 128;                 // 16 rows x 2 halves x 128 B

struct DecSmem {
  static constexpr uint32_t stages = 0;
  static constexpr uint32_t q = stages + kDecStages * kDecStageBytes;
  static constexpr uint32_t bars = q + kDecQBytes;       // full[kDecMaxStages], empty[kDecMaxStages]
  static constexpr uint32_t misc = bars + 2 * kDecMaxStages * 8;
  static constexpr uint32_t ml = misc + 16;              // [4 warps][16 rows][2] floats
  static constexpr uint32_t total = ml + 4 * 16 * 2 * 4;
};
constexpr uint32_t kDecSmemBytes = DecSmem::total + 1024;

struct DecRange {
  int s0, s1;  // keys of this split
};

__device__ __forceinline__ DecRange split_range(const DecodeParams& p, int b, int split) {
  const int L = min(max(p.seq_lens[b], 0), p.Smax);
  const int lo = p.route[b] != 0 ? 0 : max(0, L - p.window);
  const int s0 = lo + split * p.split_keys;
  return DecRange{s0, min(L, s0 + p.split_keys)};
}

// kFp8: the K/V cache holds FP8 e4m3 with per-(b, KV head) scales; the products
// then run in FP16 (Q, the converted K/V and P), exact for the e4m3 inputs.
template <bool kFp8>
__global__ void __launch_bounds__(kDecThreads, 3) switch_decode_kernel(const __grid_constant__ DecodeParams p) {
  const int split = blockIdx.x;
  const int g = blockIdx.y / p.nhb;
  const int hb = blockIdx.y % p.nhb;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t part = ((static_cast<int64_t>(b) * p.Hkv + g) * p.nhb + hb) * p.splits + split;
  float* po = p.part_o + part * 16 * 128;
  float* pml = p.part_ml + part * 16 * 2;
  const DecRange rg = split_range(p, b, split);
  if (rg.s1 <= rg.s0) {  // nothing of this sequence falls in this split (the merge skips its O)
    if (threadIdx.x < 16) {
      pml[2 * threadIdx.x] = -INFINITY;
      pml[2 * threadIdx.x + 1] = 0.0f;
    }
    return;
  }
  const int ntiles = (rg.s1 - rg.s0 + kDecTileKeys - 1) / kDecTileKeys;

  extern __shared__ uint8_t dsm_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int kSt = kFp8 ? kDecStages8 : kDecStages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + DecSmem::bars);
  uint64_t* empty = full + kDecMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + DecSmem::misc);
  float* ml = reinterpret_cast<float*>(smem + DecSmem::ml);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSt; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // Q head block into shared memory (two 64-dim halves, 128B swizzle): thread t
  // copies 16-byte chunks; rows of heads past r are zero.  The FP8 path builds its
  // Q fragments from global memory instead.
  const int head0 = g * p.r + hb * 16;
  for (int i = threadIdx.x; !kFp8 && i < 16 * 16; i += kDecThreads) {
    const int row = i >> 4, c = i & 15;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (hb * 16 + row < p.r)
      val = *reinterpret_cast<const uint4*>(p.q + (static_cast<int64_t>(b) * p.Hq + head0 + row) * 128 + 8 * c);
    *reinterpret_cast<uint4*>(smem + DecSmem::q + swz(16, row, c)) = val;
  }
  __syncthreads();

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&p.k_map);
      tma_prefetch_desc(&p.v_map);
      int t = 0;
      for (; t < ntiles; ++t) {
        const int s = t % kSt;
        if (!mbar_wait(&empty[s], ((t / kSt) & 1) ^ 1, abort_flag)) break;
        const int key0 = rg.s0 + t * kDecTileKeys;
        if constexpr (kFp8) {
          mbar_arrive_expect_tx(&full[s], kDecStageBytes8);
          uint8_t* dst = smem + DecSmem::stages + s * kDecStageBytes8;
          tma_load_4d(dst, &p.k_map, &full[s], 0, g, key0, b);
          tma_load_4d(dst + kDecTileKeys * 128, &p.v_map, &full[s], 0, g, key0, b);
        } else {
          mbar_arrive_expect_tx(&full[s], kDecStageBytes);
          uint8_t* dst = smem + DecSmem::stages + s * kDecStageBytes;
          tma_load_4d(dst, &p.k_map, &full[s], 0, g, key0, b);
          tma_load_4d(dst + kDecHalfBytes, &p.k_map, &full[s], 64, g, key0, b);
          tma_load_4d(dst + 2 * kDecHalfBytes, &p.v_map, &full[s], 0, g, key0, b);
          tma_load_4d(dst + 3 * kDecHalfBytes, &p.v_map, &full[s], 64, g, key0, b);
        }
      }
      if (*abort_flag) {
        // let the loads already issued land before the CTA's shared memory is released
        for (int u = max(0, t - kSt); u < t; ++u) {
          volatile int dummy = 0;
          mbar_wait(&full[u % kSt], (u / kSt) & 1, &dummy);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ math warps
    const uint32_t q_base = smem_u32(smem + DecSmem::q);
    const int qr = lane >> 2;          // rows qr and qr + 8 of the head block
    const int qc = 2 * (lane & 3);     // columns qc, qc + 1 of each 8-wide n tile
    uint32_t qa[8][4];  // A fragments of the 16 x 128 Q block, one per 16-dim k step
    if constexpr (kFp8) {
      // FP16, with the k slots of each 16-dim step in the order the byte tiles give
      // the K fragments: slots (2j, 2j + 1) = dims (4j, 4j + 1), slots (2j + 8,
      // 2j + 9) = dims (4j + 2, 4j + 3), j = lane % 4
      const int j = lane & 3;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int row = qr + 8 * hr;
          uint2 w = make_uint2(0, 0);
          if (hb * 16 + row < p.r)
            w = *reinterpret_cast<const uint2*>(p.q + (static_cast<int64_t>(b) * p.Hq + head0 + row) * 128 +
                                                16 * ks + 4 * j);
          qa[ks][hr] = pack_f16x2(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xFFFF0000u));
          qa[ks][2 + hr] = pack_f16x2(__uint_as_float(w.y << 16), __uint_as_float(w.y & 0xFFFF0000u));
        }
      }
    } else {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int mat = lane >> 3;
        const int row = (mat & 1) * 8 + (lane & 7);
        const int c = 2 * ks + (mat >> 1);
        ldsm_x4(q_base + swz(16, row, c), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
      }
    }
    float m[2] = {-INFINITY, -INFINITY};
    float l[2] = {0.0f, 0.0f};
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    const float sl2 = kFp8 ? p.scale_log2 * p.k_scale[b * p.Hkv + g] : p.scale_log2;
    const int klo = p.route[b] != 0 ? 0 : max(0, min(max(p.seq_lens[b], 0), p.Smax) - p.window);
    const int khi = rg.s1;
    for (int t = 0; t < ntiles; ++t) {
      const int s = t % kSt;
      if (!mbar_wait(&full[s], (t / kSt) & 1, abort_flag)) break;
      const uint32_t kb = kFp8 ? smem_u32(smem + DecSmem::stages + s * kDecStageBytes8)
                               : smem_u32(smem + DecSmem::stages + s * kDecStageBytes);
      const uint32_t vb = kFp8 ? kb + kDecTileKeys * 128 : kb + 2 * kDecHalfBytes;
      // S = Q K^T for this warp's 16 keys (two n tiles of 8)
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      if constexpr (kFp8) {
        // one ldmatrix.x4 on the byte tile (8 keys x 16 bytes per matrix): matrices
        // (keys 0-7, step ks), (0-7, ks + 1), (8-15, ks), (8-15, ks + 1) of this warp's
        // keys; lane l gets bytes 4 (l % 4) .. + 3 of key l / 4, i.e. dims 4j .. 4j + 3
        // of the step, two FP16 pairs = the B fragment in the permuted k order of qa
#pragma unroll
        for (int ks = 0; ks < 8; ks += 2) {
          const int mat = lane >> 3;
          const int key = 16 * warp + (mat >> 1) * 8 + (lane & 7);
          const int c = ks + (mat & 1);
          uint32_t r[4], bl[4], bh[4];
          ldsm_x4(kb + key * 128 + ((c ^ (key & 7)) << 4), r[0], r[1], r[2], r[3]);
#pragma unroll
          for (int e = 0; e < 4; ++e) e4m3x4_to_f16x2x2(r[e], bl[e], bh[e]);
          mma_f16(sc[0], qa[ks], bl[0], bh[0]);
          mma_f16(sc[1], qa[ks], bl[2], bh[2]);
          mma_f16(sc[0], qa[ks + 1], bl[1], bh[1]);
          mma_f16(sc[1], qa[ks + 1], bl[3], bh[3]);
        }
      } else {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int mat = lane >> 3;
          const int key = 16 * warp + (mat >> 1) * 8 + (lane & 7);
          const int c = 2 * ks + (mat & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kb + swz(kDecTileKeys, key, c), b0, b1, b2, b3);
          mma_bf16(sc[0], qa[ks], b0, b1);
          mma_bf16(sc[1], qa[ks], b2, b3);
        }
      }
      // mask, online softmax (rows qr, qr + 8)
      const int key0 = rg.s0 + t * kDecTileKeys + 16 * warp;
      float mx[2] = {-INFINITY, -INFINITY};
      if (key0 >= klo && key0 + 16 <= khi) {  // every key of the warp legal (warp-uniform)
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            sc[n][e] *= sl2;
            mx[e >> 1] = fmaxf(mx[e >> 1], sc[n][e]);
          }
      } else {
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = key0 + 8 * n + qc + (e & 1);
            const float x = (key >= klo && key < khi) ? sc[n][e] * sl2 : -INFINITY;
            sc[n][e] = x;
            mx[e >> 1] = fmaxf(mx[e >> 1], x);
          }
      }
      // The running max is only raised (and O, l rescaled) when the tile's max
      // exceeds it by more than kDecRescale: the (max, sum, O) triple stays
      // consistent, so the merged result is the same, and P stays below 2^kDecRescale.
      bool grow[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        grow[h] = mx[h] > m[h] + kDecRescale;  // false while both are -inf
      }
      if (__any_sync(0xffffffffu, grow[0] || grow[1])) {
        float alpha[2] = {1.0f, 1.0f};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (grow[h]) {
            alpha[h] = ex2_approx(m[h] - mx[h]);  // 0 for the first legal tile (m = -inf)
            m[h] = mx[h];
            l[h] *= alpha[h];
          }
        }
        // O of earlier tiles to the new running maximum
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          o[n][0] *= alpha[0];
          o[n][1] *= alpha[0];
          o[n][2] *= alpha[1];
          o[n][3] *= alpha[1];
        }
      }
      uint32_t pa[4];
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        float pv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mh = m[e >> 1];
          pv[e] = (mh == -INFINITY) ? 0.0f : ex2_approx(sc[n][e] - mh);
          l[e >> 1] += pv[e];
        }
        if constexpr (kFp8) {
          pa[2 * n] = pack_f16x2(pv[0], pv[1]);
          pa[2 * n + 1] = pack_f16x2(pv[2], pv[3]);
        } else {
          pa[2 * n] = pack_bf16x2(pv[0], pv[1]);
          pa[2 * n + 1] = pack_bf16x2(pv[2], pv[3]);
        }
      }
      // O += P V: P (16 rows x 16 keys) as the A fragment, V via transposed ldmatrix
      const uint32_t a[4] = {pa[0], pa[1], pa[2], pa[3]};
      if constexpr (kFp8) {
        // ldmatrix.x4.trans on the byte tile: matrices (keys 0-7, 16-dim chunk cc),
        // (8-15, cc), (0-7, cc + 1), (8-15, cc + 1); lane l gets keys 2j, 2j + 1 (j =
        // l % 4) of dims 16 cc + 2 (l / 4) and + 1 as bytes [k0 d0, k0 d1, k1 d0, k1 d1].
        // The (k0, k1) byte pairs of d0 and of d1 are the B fragments of two MMAs whose
        // n slots are the even and the odd dims of the chunk: o[2 cc] and o[2 cc + 1]
        // (output column of o[n][e]: out_col below).
#pragma unroll
        for (int cc = 0; cc < 8; cc += 2) {
          const int mat = lane >> 3;
          const int key = 16 * warp + (mat & 1) * 8 + (lane & 7);
          const int c = cc + (mat >> 1);
          uint32_t r0, r1, r2, r3;
          ldsm_x4_t(vb + key * 128 + ((c ^ (key & 7)) << 4), r0, r1, r2, r3);
          const uint32_t rr[4] = {r0, r1, r2, r3};
          uint32_t ev[4], od[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint32_t k0, k1;  // (k0 d0, k0 d1), (k1 d0, k1 d1)
            e4m3x4_to_f16x2x2(rr[e], k0, k1);
            ev[e] = __byte_perm(k0, k1, 0x5410);
            od[e] = __byte_perm(k0, k1, 0x7632);
          }
          mma_f16(o[2 * cc], a, ev[0], ev[1]);
          mma_f16(o[2 * cc + 1], a, od[0], od[1]);
          mma_f16(o[2 * cc + 2], a, ev[2], ev[3]);
          mma_f16(o[2 * cc + 3], a, od[2], od[3]);
        }
      } else {
#pragma unroll
        for (int nd = 0; nd < 16; nd += 2) {
          const int mat = lane >> 3;
          const int key = 16 * warp + (mat & 1) * 8 + (lane & 7);
          const int c = nd + (mat >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vb + swz(kDecTileKeys, key, c), b0, b1, b2, b3);
          mma_bf16(o[nd], a, b0, b1);
          mma_bf16(o[nd + 1], a, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // row sums over the quad
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
      l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
    }
    if ((lane & 3) == 0) {
      ml[(warp * 16 + qr) * 2] = m[0];
      ml[(warp * 16 + qr) * 2 + 1] = l[0];
      ml[(warp * 16 + qr + 8) * 2] = m[1];
      ml[(warp * 16 + qr + 8) * 2 + 1] = l[1];
    }
    named_bar_sync(1, 128);
    // A warp that gave up a wait set the flag before this barrier, so all four
    // agree.  Then loads may still be landing in the ring: leave it alone.
    if (*abort_flag) goto done;
    {
    // merge the four warps: scale to the block maximum, sum into the partial
    float f[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = qr + 8 * h;
      float mc = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) mc = fmaxf(mc, ml[(w * 16 + row) * 2]);
      f[h] = (m[h] == -INFINITY) ? 0.0f : ex2_approx(m[h] - mc);
      if constexpr (kFp8) f[h] *= p.v_scale[b * p.Hkv + g];  // O of the FP8 values -> O of K/V x scale
      if (warp == 0 && (lane & 3) == 0) {
        float lc = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float mw = ml[(w * 16 + row) * 2];
          lc += (mw == -INFINITY) ? 0.0f : ml[(w * 16 + row) * 2 + 1] * ex2_approx(mw - mc);
        }
        pml[2 * row] = mc;
        pml[2 * row + 1] = lc;
      }
    }
    // the ring is drained: reuse stage memory as a [16][128] FP32 accumulator
    float* acc = reinterpret_cast<float*>(smem + DecSmem::stages);
    for (int i = threadIdx.x; i < 16 * 128; i += 128) acc[i] = 0.0f;
    named_bar_sync(1, 128);
    // output column of accumulator o[n][e] (e = 0, 1; e = 2, 3 the same for row qr + 8):
    // BF16 path 8 n + qc + e; FP8 path chunk n / 2, parity n % 2 (even / odd dims):
    // 16 (n / 2) + 2 qc + 2 e + n % 2
    auto out_col = [&](int n, int e) { return kFp8 ? 16 * (n >> 1) + 2 * qc + 2 * e + (n & 1) : 8 * n + qc + e; };
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      atomicAdd(&acc[qr * 128 + out_col(n, 0)], o[n][0] * f[0]);
      atomicAdd(&acc[qr * 128 + out_col(n, 1)], o[n][1] * f[0]);
      atomicAdd(&acc[(qr + 8) * 128 + out_col(n, 0)], o[n][2] * f[1]);
      atomicAdd(&acc[(qr + 8) * 128 + out_col(n, 1)], o[n][3] * f[1]);
    }
    named_bar_sync(1, 128);
    const int rows = min(16, p.r - hb * 16);  // head rows that exist
    for (int i = threadIdx.x; i < rows * 128 / 4; i += 128)
      reinterpret_cast<float4*>(po)[i] = reinterpret_cast<const float4*>(acc)[i];
    }
  }
done:
  if (threadIdx.x == 0 && *abort_flag) atomicOr(p.status, kStatusTimeout);
}

// Merge the splits of one (batch, KV group, head block): O = sum_s O_s 2^(m_s - M) / L,
// L = sum_s l_s 2^(m_s - M), LSE = log2 L + M (log2 units, as the prefill path).
__global__ void __launch_bounds__(128) switch_decode_combine_kernel(const __grid_constant__ DecodeParams p) {
  const int g = blockIdx.x / p.nhb;
  const int hb = blockIdx.x % p.nhb;
  const int b = blockIdx.y;
  const int64_t part0 = ((static_cast<int64_t>(b) * p.Hkv + g) * p.nhb + hb) * p.splits;
  __shared__ float sM[16], sL[16];
  if (threadIdx.x < 16) {
    const int row = threadIdx.x;
    float M = -INFINITY;
    for (int s = 0; s < p.splits; ++s) M = fmaxf(M, p.part_ml[((part0 + s) * 16 + row) * 2]);
    float L = 0.0f;
    for (int s = 0; s < p.splits; ++s) {
      const float ms = p.part_ml[((part0 + s) * 16 + row) * 2];
      if (ms != -INFINITY) L += p.part_ml[((part0 + s) * 16 + row) * 2 + 1] * ex2_approx(ms - M);
    }
    sM[row] = M;
    sL[row] = L;
    const int h = hb * 16 + row;
    if (h < p.r) p.lse[static_cast<int64_t>(b) * p.Hq + g * p.r + h] = lg2_approx(L) + M;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * 64; i += 128) {  // pairs of columns
    const int row = i >> 6, c2 = (i & 63) * 2;
    const int h = hb * 16 + row;
    if (h >= p.r) continue;
    float a0 = 0.0f, a1 = 0.0f;
    for (int s = 0; s < p.splits; ++s) {
      const float ms = p.part_ml[((part0 + s) * 16 + row) * 2];
      if (ms == -INFINITY) continue;
      const float w = ex2_approx(ms - sM[row]);
      const float2 v = *reinterpret_cast<const float2*>(p.part_o + ((part0 + s) * 16 + row) * 128 + c2);
      a0 += v.x * w;
      a1 += v.y * w;
    }
    const float inv = 1.0f / sL[row];
    *reinterpret_cast<uint32_t*>(p.out + (static_cast<int64_t>(b) * p.Hq + g * p.r + h) * 128 + c2) =
        pack_bf16x2(a0 * inv, a1 * inv);
  }
}

}  // namespace

uint32_t decode_smem_bytes() { return kDecSmemBytes; }

cudaError_t launch_decode(const DecodeParams& params, cudaStream_t stream) {
  static bool attr_set[2][64] = {};
  const int f8 = params.fp8 != 0 ? 1 : 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[f8][dev]) {
    cudaError_t e = f8 ? cudaFuncSetAttribute(switch_decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kDecSmemBytes)
                       : cudaFuncSetAttribute(switch_decode_kernel<false>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, kDecSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set[f8][dev] = true;
  }
  const dim3 grid(params.splits, params.Hkv * params.nhb, params.B);
  if (f8) {
    switch_decode_kernel<true><<<grid, kDecThreads, kDecSmemBytes, stream>>>(params);
  } else {
    switch_decode_kernel<false><<<grid, kDecThreads, kDecSmemBytes, stream>>>(params);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  switch_decode_combine_kernel<<<dim3(params.Hkv * params.nhb, params.B), 128, 0, stream>>>(params);
  return cudaGetLastError();
}

}  // namespace swa
