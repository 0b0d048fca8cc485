// Switch Attention GQA prefill backward (sm_100a): dQ, dK, dV from the forward's
// output O and log2-domain LSE, for both routing branches.  The reference is
// forward only (swiattn_gqa_prefill_varlen.py:14); the gradients are those of
// its forward: P = 2^(S * scale_log2 - LSE) over the row's legal keys (masks
// swiattn_gqa_prefill.py:145-158, varlen bounds swiattn_gqa_prefill_varlen.py:186-196),
// dP = dO V^T, dS = P (dP - D) with D = rowsum(dO * O), dQ = scale dS K,
// dK = scale dS^T Q, dV = P^T dO.
//
// Rows are packed as in the forward: packed row R of (branch, batch b, KV group
// g) is routed slot R / r of the branch's list and query head g r + R % r, so
// the r heads that share K/V sit in one matrix dimension and dK / dV sum over
// them inside the matrix products.
//   bwd_pack_kernel  : half a warp per packed row: Q and dO copied into packed
//                      order, the row's record {lo, hi, LSE, D} and position,
//                      so both passes read contiguous rows without index chains.
//   bwd_dq_tc_kernel : one CTA per 128 packed rows; loops over the 64-key tiles
//                      of the rows' union key range: S = Q K^T and dP = dO V^T,
//                      dS, dQ += dS K, on tcgen05 (see its comment below).
//   bwd_dkv_tc_kernel: one CTA per 128-key tile; loops over the packed rows
//                      whose key range meets the tile (a slot range per branch,
//                      found by binary search in the sorted index lists), 64 at
//                      a time, on tcgen05 (see its comment below).
// Both passes take BF16 operands with FP32 accumulation in TMEM; P and dS are
// rounded to BF16 where they are operands of a product.
#include "sm100.cuh"
#include "swattn_internal.h"

namespace swa {

namespace {

__device__ __forceinline__ void bwd_row_bounds(const BwdParams& p, int branch, int pos, int& lo, int& hi) {
  if (p.ends != nullptr) {
    lo = max(p.starts[branch][pos], 0);
    hi = min(p.ends[pos], p.Skv);
  } else {
    lo = branch ? max(pos - p.window + 1, 0) : 0;
    hi = min(pos + 1, p.Skv);
  }
}

__device__ __forceinline__ float2 bf2_to_f2(uint32_t u) {
  __nv_bfloat162 h;
  memcpy(&h, &u, 4);
  return __bfloat1622float2(h);
}

// First packed row of (branch, b, g).
__device__ __forceinline__ int64_t packed_base(const BwdParams& p, int branch, int b, int g) {
  return (branch ? p.pk_n0 : 0) + (static_cast<int64_t>(b) * p.Hkv + g) * p.idx_stride[branch] * p.r;
}

// Half a warp per packed row (16 bytes per lane); 32-bit index arithmetic (the
// host bounds the packed rows below 2^31).
__global__ void __launch_bounds__(256) bwd_pack_kernel(const __grid_constant__ BwdParams p) {
  const int hl = threadIdx.x & 15;
  const uint32_t hmask = 0xffffu << (threadIdx.x & 16);
  const int n0 = static_cast<int>(p.pk_n0), nrows = static_cast<int>(p.pk_rows);
  const int stride = gridDim.x * (blockDim.x >> 4);
  for (int pr = (blockIdx.x * blockDim.x + threadIdx.x) >> 4; pr < nrows; pr += stride) {
    const int branch = pr < n0 ? 0 : 1;
    const int local = branch ? pr - n0 : pr;
    const int per = p.idx_stride[branch] * p.r;
    const int bg = local / per;
    const int R = local - bg * per;
    const int g = bg % p.Hkv, b = bg / p.Hkv;
    const int cnt = min(p.counts[2 * b + branch], p.idx_stride[branch]);
    const int slot = R / p.r;
    int pos = -1;
    if (slot < cnt) {
      pos = p.idx[branch][static_cast<int64_t>(b) * p.idx_stride[branch] + slot];
      if (pos < 0 || pos >= p.Sq) pos = -1;
    }
    uint4 qv = make_uint4(0, 0, 0, 0), dv = make_uint4(0, 0, 0, 0);
    int4 rec = make_int4(0, 0, 0, 0);
    if (pos >= 0) {  // (uniform in the half-warp)
      const int64_t row = (static_cast<int64_t>(b) * p.Sq + pos) * p.Hq + g * p.r + R % p.r;
      qv = *reinterpret_cast<const uint4*>(p.q + row * 128 + 8 * hl);
      dv = *reinterpret_cast<const uint4*>(p.dout + row * 128 + 8 * hl);
      const uint4 o = *reinterpret_cast<const uint4*>(p.o + row * 128 + 8 * hl);
      float d = 0.0f;
      const uint32_t da[4] = {dv.x, dv.y, dv.z, dv.w}, oa[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = bf2_to_f2(da[i]), c = bf2_to_f2(oa[i]);
        d += a.x * c.x + a.y * c.y;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) d += __shfl_xor_sync(hmask, d, off);
      int lo, hi;
      bwd_row_bounds(p, branch, pos, lo, hi);
      float lse = p.lse[row];
      if (!(lse > -INFINITY)) {
        // a row without legal keys (forward O = NaN, LSE = -inf) has no gradient:
        // empty key range, and finite LSE / D so that no NaN reaches its masked entries
        hi = lo;
        lse = 0.0f;
        d = 0.0f;
      }
      rec = make_int4(lo, max(hi, lo), __float_as_int(lse), __float_as_int(d));
    }
    *reinterpret_cast<uint4*>(p.qp + static_cast<int64_t>(pr) * 128 + 8 * hl) = qv;
    *reinterpret_cast<uint4*>(p.dop + static_cast<int64_t>(pr) * 128 + 8 * hl) = dv;
    if (hl == 0) {
      p.rec[pr] = rec;
      p.rpos[pr] = pos;
    }
  }
}

// First slot in [0, cnt) whose row satisfies pred (monotone: false...true), or
// cnt; the 32 lanes of a warp probe 32 points per round, so a list of 32^k slots
// takes k rounds of one load each.  Warp-collective; every lane gets the result.
template <typename Pred>
__device__ __forceinline__ int first_slot_warp(int cnt, Pred pred) {
  const int lane = threadIdx.x & 31;
  int lo = 0, hi = cnt;
  while (lo < hi) {
    const int n = hi - lo;
    const int s = lo + static_cast<int>((static_cast<int64_t>(n) * lane) >> 5);
    const uint32_t m = __ballot_sync(0xffffffffu, pred(s));
    if (m == 0u) {
      lo = __shfl_sync(0xffffffffu, s, 31) + 1;
    } else {
      const int f = __ffs(m) - 1;
      const int sf = __shfl_sync(0xffffffffu, s, f);
      const int sp = __shfl_sync(0xffffffffu, s, f > 0 ? f - 1 : 0);
      hi = sf;
      lo = f > 0 ? sp + 1 : hi;
    }
  }
  return lo;
}

// A bounded wait whose outcome is the same in every lane of the warp (the
// warp-collective tcgen05 instructions after it need the whole warp).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
}

// ---------------------------------------------------------------------------
// dK / dV pass on the 5th-generation tensor cores.  One CTA per 128-key tile of
// (b, g), 320 threads, over blocks of 64 packed rows:
//   warp 0     TMA: the CTA's K and V tiles once, then per block the rows' Q and
//              dO tiles and records (consecutive packed rows: one box each) into
//              a 4-entry ring.
//   warp 1     MMA: per block t, S^T = K Q^T and dP^T = V dO^T (SS, N = 64, both
//              K-major) into TMEM buffer t & 1; then, once P^T / dS^T of block
//              t - 1 are in TMEM, dV += P^T dO and dK += dS^T Q (TS, dO / Q
//              MN-major), whose commit frees ring entry t - 1.  The products of
//              block t + 1 thus run while the elementwise warps work on block t.
//   warps 2-17 elementwise, two groups of eight taking alternate blocks (group
//              g the blocks t with t & 1 == g, i.e. TMEM buffer g), so one
//              group's TMEM round trips and waits overlap the other's arithmetic.
//              In a group, two threads per key (TMEM lane = key), 32 rows each, in
//              two 16-row chunks: P^T = 2^(S^T scale_log2 - LSE_row) on the legal
//              entries, dS^T = P^T (dP^T - D_row), written as BF16 pairs over the
//              thread's own, already read S^T / dP^T columns.  Group 0 then
//              writes dK, group 1 dV.
// A block starts at a slot-range row of its branch and may run past the range's
// end into later rows (of this or the next (b, g)): those rows are masked by
// their index in the block, whatever their records say.
// TMEM: S^T[2] | dP^T[2] (64 columns each) | dV | dK.
constexpr int kTcKeys = 128;
constexpr int kTcRows = 64;
constexpr int kTcStages = 4;
constexpr int kTcThreads = 576;
constexpr uint32_t kTcKvTile = 128 * 256;   // 128 keys x 128 dims BF16 (two 16 KB halves)
constexpr uint32_t kTcRowTile = 64 * 256;   // 64 rows x 128 dims BF16 (two 8 KB halves)
constexpr uint32_t kTcRecBytes = kTcRows * 16;

struct TcSmem {
  static constexpr uint32_t k = 0;
  static constexpr uint32_t v = k + kTcKvTile;
  static constexpr uint32_t stage = v + kTcKvTile;                        // kTcStages x (Q, dO, records)
  static constexpr uint32_t stage_bytes = 2 * kTcRowTile + kTcRecBytes;   // 33 KB (1024-byte multiple)
  static constexpr uint32_t bars = stage + kTcStages * stage_bytes;      // kv, full[4], empty[4], s_full[2], p_full[2], done
  static constexpr uint32_t misc = bars + 16 * 8;                         // tmem holder, abort flag, slot ranges
  static constexpr uint32_t total = misc + 64;
};
static_assert(TcSmem::stage_bytes % 1024 == 0, "ring entries keep the 1024-byte alignment of the swizzled tiles");
constexpr uint32_t kTcSmemBytes = TcSmem::total + 1024;

__global__ void __launch_bounds__(kTcThreads, 1) bwd_dkv_tc_kernel(const __grid_constant__ BwdParams p) {
  const int k0 = blockIdx.x * kTcKeys, g = blockIdx.y, b = blockIdx.z;
  extern __shared__ uint8_t bsm_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(bsm_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcSmem::bars);
  uint64_t* kv_full = bars;
  uint64_t* full = bars + 1;                   // [kTcStages]
  uint64_t* empty = full + kTcStages;          // [kTcStages]
  uint64_t* s_full = empty + kTcStages;        // [2]
  uint64_t* p_full = s_full + 2;               // [2]
  uint64_t* done = p_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + TcSmem::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + TcSmem::misc + 4);
  int* ranges = reinterpret_cast<int*>(smem + TcSmem::misc + 8);  // first slot [2], end slot [2] per branch
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 256);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp < 4) {
    // rows of each branch whose key range [lo, hi) meets [k0, k0 + 128): a slot range,
    // both bounds being non-decreasing along the increasing routed positions.
    // Warp w finds bound w & 1 of branch w >> 1.
    __syncwarp();
    const int branch = warp >> 1;
    const int cnt = min(p.counts[2 * b + branch], p.idx_stride[branch]);
    const int32_t* idx = p.idx[branch] + static_cast<int64_t>(b) * p.idx_stride[branch];
    auto bounds = [&](int slot, int& lo, int& hi) {
      const int pos = min(max(idx[min(slot, cnt - 1)], 0), p.Sq - 1);
      bwd_row_bounds(p, branch, pos, lo, hi);
    };
    const int found = (warp & 1) == 0
        ? first_slot_warp(cnt, [&](int s) { int lo, hi; bounds(s, lo, hi); return hi > k0; })
        : first_slot_warp(cnt, [&](int s) { int lo, hi; bounds(s, lo, hi); return lo >= k0 + kTcKeys; });
    if (lane == 0) ranges[2 * (warp & 1) + branch] = found;
  }
  if (warp == 0) {
    __syncwarp();  // tcgen05.alloc is warp-collective: lane 0 comes from the set-up above
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // slot ranges, re-read from shared memory where needed (registers are scarce)
  auto branch_blocks = [&](int br) {
    return ((max(ranges[br], ranges[2 + br]) - ranges[br]) * p.r + kTcRows - 1) / kTcRows;
  };
  const int nblocks = branch_blocks(0) + branch_blocks(1);
  const uint32_t tm_dv = tmem + 256, tm_dk = tmem + 384;
  auto tm_st = [&](int t) { return tmem + 64 * (t & 1); };
  auto tm_dpt = [&](int t) { return tmem + 128 + 64 * (t & 1); };
  // block it: rows [R0, R0 + 64) of its branch, the first `valid` of them in the slot range
  auto block_rows = [&](int it, int& branch, int& R0, int& valid) {
    const int nb0 = branch_blocks(0);
    branch = it < nb0 ? 0 : 1;
    const int t = branch ? it - nb0 : it;
    const int s_lo = ranges[branch];
    R0 = s_lo * p.r + t * kTcRows;
    valid = min(kTcRows, max(s_lo, ranges[2 + branch]) * p.r - R0);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && nblocks > 0) {
      tma_prefetch_desc(&p.k_map);
      tma_prefetch_desc(&p.v_map);
      tma_prefetch_desc(&p.qp_map);
      tma_prefetch_desc(&p.dop_map);
      tma_prefetch_desc(&p.rec_map);
      // the K and V tiles: per 64-dim half, keys k0 .. k0 + 63 and k0 + 64 .. k0 + 127
      // (zeros past Skv)
      mbar_arrive_expect_tx(kv_full, 2 * kTcKvTile);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint32_t off = h * (kTcKvTile / 2) + kk * (kTcKvTile / 4);
          tma_load_4d(smem + TcSmem::k + off, &p.k_map, kv_full, 64 * h, g, k0 + 64 * kk, b);
          tma_load_4d(smem + TcSmem::v + off, &p.v_map, kv_full, 64 * h, g, k0 + 64 * kk, b);
        }
      }
      int it = 0;
      for (; it < nblocks; ++it) {
        const int s = it % kTcStages;
        if (!mbar_wait(&empty[s], ((it / kTcStages) & 1) ^ 1, abort_flag)) break;
        int branch, R0, valid;
        block_rows(it, branch, R0, valid);
        const int pr0 = static_cast<int>(packed_base(p, branch, b, g) + R0);
        uint8_t* st = smem + TcSmem::stage + s * TcSmem::stage_bytes;
        mbar_arrive_expect_tx(&full[s], TcSmem::stage_bytes);
        tma_load_2d(st, &p.qp_map, &full[s], 0, pr0);
        tma_load_2d(st + kTcRowTile / 2, &p.qp_map, &full[s], 64, pr0);
        tma_load_2d(st + kTcRowTile, &p.dop_map, &full[s], 0, pr0);
        tma_load_2d(st + kTcRowTile + kTcRowTile / 2, &p.dop_map, &full[s], 64, pr0);
        tma_load_2d(st + 2 * kTcRowTile, &p.rec_map, &full[s], 0, pr0);
      }
      if (*abort_flag) {
        // let the loads already issued land before the CTA's shared memory is released
        volatile int dummy = 0;
        mbar_wait(kv_full, 0, &dummy);
        for (int u = max(0, it - kTcStages); u < it; ++u) mbar_wait(&full[u % kTcStages], (u / kTcStages) & 1, &dummy);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 64, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, 128, false, true);
    const uint64_t k_desc = make_smem_desc_sw128(smem_u32(smem + TcSmem::k), 16, 1024);
    const uint64_t v_desc = make_smem_desc_sw128(smem_u32(smem + TcSmem::v), 16, 1024);
    auto products = [&](int t) {  // dV += P^T dO, dK += dS^T Q of block t
      const int s = t % kTcStages;
      const uint32_t qa = smem_u32(smem + TcSmem::stage + s * TcSmem::stage_bytes), doa = qa + kTcRowTile;
      const uint64_t do_mn = make_smem_desc_sw128(doa, kTcRowTile / 2, 1024);
      const uint64_t q_mn = make_smem_desc_sw128(qa, kTcRowTile / 2, 1024);
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // rows 32 c .. 32 c + 31: BF16 pairs in columns 32 c .. 32 c + 15
        const uint32_t acc = (t > 0 || c > 0) ? 1u : 0u;
        umma_ts_k32_warp(tm_dv, tm_st(t) + 32 * c, do_mn + 2 * c * 128, idesc_o, acc);
        umma_ts_k32_warp(tm_dk, tm_dpt(t) + 32 * c, q_mn + 2 * c * 128, idesc_o, acc);
      }
      tc_commit_warp(&empty[s]);
    };
    bool ok = nblocks == 0 || warp_wait(kv_full, 0, abort_flag);
    for (int it = 0; it < nblocks && ok; ++it) {
      const int s = it % kTcStages;
      if (!warp_wait(&full[s], (it / kTcStages) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      // TMEM buffer it & 1 was last read by the products of block it - 2, issued earlier
      const uint32_t qa = smem_u32(smem + TcSmem::stage + s * TcSmem::stage_bytes), doa = qa + kTcRowTile;
      umma_ss_k128_bhalf8k_warp(tm_st(it), k_desc, make_smem_desc_sw128(qa, 16, 1024), idesc_s);
      umma_ss_k128_bhalf8k_warp(tm_dpt(it), v_desc, make_smem_desc_sw128(doa, 16, 1024), idesc_s);
      tc_commit_warp(&s_full[it & 1]);
      if (it >= 1) {
        if (!warp_wait(&p_full[(it - 1) & 1], ((it - 1) >> 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        products(it - 1);
      }
    }
    if (ok && nblocks >= 1) {
      const int t = nblocks - 1;
      if (warp_wait(&p_full[t & 1], (t >> 1) & 1, abort_flag)) {
        tc_fence_after();
        products(t);
      }
    }
    // all MMAs complete before the epilogue reads (and before the CTA frees TMEM)
    tc_commit_warp(done);
  } else {
    // ------------------------------------------------------------ elementwise + epilogue
    const int ew = warp - 2;
    const int grp = ew >> 3;           // blocks t with (t & 1) == grp
    const int quarter = warp & 3;
    const int half = (ew >> 2) & 1;    // rows 32 half .. 32 half + 31 of a block
    const int key = k0 + 32 * quarter + lane;
    const uint32_t lane_off = static_cast<uint32_t>(32 * quarter) << 16;
    const float sl2 = p.scale_log2;
    bool ok = true;
    for (int it = grp; it < nblocks; it += 2) {
      const int s = it % kTcStages, tb = it & 1;
      int branch, R0, valid;
      block_rows(it, branch, R0, valid);
      if (!warp_wait(&s_full[tb], (it >> 1) & 1, abort_flag)) { ok = false; break; }
      // (already complete: makes the records the TMA wrote visible to this thread)
      if (!warp_wait(&full[s], (it / kTcStages) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int4* rec = reinterpret_cast<const int4*>(smem + TcSmem::stage + s * TcSmem::stage_bytes + 2 * kTcRowTile);
      // every entry of the warp legal (its 32 keys inside each of its 32 rows' ranges,
      // all rows in the block's slot range): no masking.  Lane j checks row j.
      const int4 mine = rec[32 * half + lane];
      const int kmin = k0 + 32 * quarter;
      const bool all_legal =
          __all_sync(0xffffffffu, 32 * half + lane < valid && mine.x <= kmin && mine.y >= kmin + 32);
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // rows 32 half + 16 c .. + 15: read columns 16 c .., write 8 c ..
        uint32_t sr[16], dr[16];
        tmem_ld_x16(tm_st(it) + lane_off + 32 * half + 16 * c, sr);
        tmem_ld_x16(tm_dpt(it) + lane_off + 32 * half + 16 * c, dr);
        tmem_ld_wait();
        reg_fence16(sr);
        reg_fence16(dr);
        uint32_t pk[8], dk2[8];
        if (all_legal) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float pv[2], dsv[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              // {LSE, D} of the row from the lane that loaded its record: warp shuffles
              // instead of shared-memory broadcasts, which the products' operand reads
              // already keep busy (+2-4 % for the backward step)
              const int src = 16 * c + 2 * j + e;
              const float2 ld = make_float2(__shfl_sync(0xffffffffu, __int_as_float(mine.z), src),
                                            __shfl_sync(0xffffffffu, __int_as_float(mine.w), src));
              pv[e] = ex2_approx(__uint_as_float(sr[2 * j + e]) * sl2 - ld.x);
              dsv[e] = pv[e] * (__uint_as_float(dr[2 * j + e]) - ld.y);
            }
            pk[j] = pack_bf16x2(pv[0], pv[1]);
            dk2[j] = pack_bf16x2(dsv[0], dsv[1]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float pv[2], dsv[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int rr = 32 * half + 16 * c + 2 * j + e;  // row of the block
              const int4 rc = rec[rr];                        // {lo, hi, LSE, D}
              const bool legal = rr < valid && key >= rc.x && key < rc.y;
              pv[e] = legal ? ex2_approx(__uint_as_float(sr[2 * j + e]) * sl2 - __int_as_float(rc.z)) : 0.0f;
              dsv[e] = pv[e] * (__uint_as_float(dr[2 * j + e]) - __int_as_float(rc.w));
            }
            pk[j] = pack_bf16x2(pv[0], pv[1]);
            dk2[j] = pack_bf16x2(dsv[0], dsv[1]);
          }
        }
        // rows 32 half .. 32 half + 31 end up as BF16 pairs in columns 32 half .. 32 half + 15
        // (chunk c over columns 32 half + 8 c .., all read before)
        tmem_st_x8(tm_st(it) + lane_off + 32 * half + 8 * c, pk);
        tmem_st_x8(tm_dpt(it) + lane_off + 32 * half + 8 * c, dk2);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[tb]);
    }
    // epilogue: group 0 dK (scaled), group 1 dV, of this thread's key, dims 64 half ..
    // 64 half + 63.  tcgen05.ld is warp-collective: every lane loads (the condition is
    // warp uniform), only the stores of keys past Skv are skipped.
    if (ok && nblocks > 0) ok = warp_wait(done, 0, abort_flag);
    tc_fence_after();
    const bool store = key < p.Skv;
    const int64_t row = (static_cast<int64_t>(b) * p.Skv + (store ? key : 0)) * p.Hkv + g;
    __nv_bfloat16* dst = (grp == 0 ? p.dk : p.dv) + row * 128 + 64 * half;
    const float sc = grp == 0 ? p.scale : 1.0f;
    const uint32_t src = (grp == 0 ? tm_dk : tm_dv) + lane_off + 64 * half;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      uint32_t r[32];
      if (nblocks > 0 && ok) {
        tmem_ld_x32(src + 32 * cc, r);
        tmem_ld_wait();
        reg_fence32(r);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
      if (store) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(r[8 * j]) * sc, __uint_as_float(r[8 * j + 1]) * sc);
          w.y = pack_bf16x2(__uint_as_float(r[8 * j + 2]) * sc, __uint_as_float(r[8 * j + 3]) * sc);
          w.z = pack_bf16x2(__uint_as_float(r[8 * j + 4]) * sc, __uint_as_float(r[8 * j + 5]) * sc);
          w.w = pack_bf16x2(__uint_as_float(r[8 * j + 6]) * sc, __uint_as_float(r[8 * j + 7]) * sc);
          *reinterpret_cast<uint4*>(dst + 32 * cc + 8 * j) = w;
        }
      }
    }
  }
  // teardown: the MMA warp's `done` commit covers every MMA it issued
  if (warp == 1) {
    volatile int dummy = 0;
    mbar_wait(done, 0, &dummy);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(p.status, kStatusTimeout);
}

// ---------------------------------------------------------------------------
// dQ pass on the 5th-generation tensor cores.  One CTA per 128 packed rows of
// (branch, b, g), 320 threads, over the 64-key tiles of the rows' union key
// range [lo of the first row, hi of the last):
//   warp 0     TMA loads of the K and V tiles (two 64-dim halves each, 128B
//              swizzle) into a 6-entry ring.
//   warp 1     MMA: per tile t, S = Q K^T and dP = dO V^T into TMEM buffer t & 1
//              (TS: Q and dO sit in TMEM, the K-major key tile is the B operand,
//              so only B is read from shared memory -- with N = 64 an SS product
//              would need more shared-memory bandwidth than the SM has); then,
//              once dS of tile t - 1 is in TMEM, dQ += dS K (TS, K MN-major),
//              whose commit frees ring entry t - 1.  The products of tile t + 1
//              thus run while the elementwise warps work on tile t.
//   warps 2-9  two threads per row (TMEM lane = row; the two 64-dim halves of
//              Q / dO, the two 32-key halves of a tile): first the row's Q and dO
//              into TMEM; per tile P = 2^(S scale_log2 - LSE) on the row's legal
//              keys and dS = P (dP - D), written as BF16 pairs over the thread's
//              own, already read dP columns; finally dQ (scaled) of the row.
// TMEM: Q | dO (64 columns each, BF16 pairs) | S[2] | dP[2] (64 each) | dQ (128).
// Full-branch blocks run latest rows first: their key ranges, and so their
// run times, grow with the position.
constexpr int kDqRows = 128;
constexpr int kDqKeys = 64;
constexpr int kDqStages = 6;
constexpr int kDqThreads = 320;
constexpr uint32_t kDqKeyTile = kDqKeys * 256;  // 64 keys x 128 dims BF16 (two 8 KB halves)

struct DqTcSmem {
  static constexpr uint32_t stage = 0;                                   // kDqStages x (K tile, V tile)
  static constexpr uint32_t bars = stage + kDqStages * 2 * kDqKeyTile;   // rows_full, full[6], empty[6], s_full[2], p_full[2], done
  static constexpr uint32_t misc = bars + 24 * 8;                        // tmem holder, abort flag, key range
  static constexpr uint32_t total = misc + 32;
};
constexpr uint32_t kDqTcSmemBytes = DqTcSmem::total + 1024;

__global__ void __launch_bounds__(kDqThreads, 1) bwd_dq_tc_kernel(const __grid_constant__ BwdParams p) {
  const int g = blockIdx.y, b = blockIdx.z;
  const int nblk0 = p.nblk[0];
  int blk = blockIdx.x, branch = 0;
  if (blk >= nblk0) {
    blk -= nblk0;
    branch = 1;
  } else {
    blk = nblk0 - 1 - blk;
  }
  const int cnt = min(p.counts[2 * b + branch], p.idx_stride[branch]);
  const int R0 = blk * kDqRows;
  if (R0 >= cnt * p.r) return;  // (the whole CTA, before any barrier or TMEM use)
  extern __shared__ uint8_t bsm_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(bsm_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DqTcSmem::bars);
  uint64_t* rows_full = bars;
  uint64_t* full = bars + 1;             // [kDqStages]
  uint64_t* empty = full + kDqStages;    // [kDqStages]
  uint64_t* s_full = empty + kDqStages;  // [2]
  uint64_t* p_full = s_full + 2;         // [2]
  uint64_t* done = p_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + DqTcSmem::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + DqTcSmem::misc + 4);
  int* range = reinterpret_cast<int*>(smem + DqTcSmem::misc + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(rows_full, 256);
    for (int s = 0; s < kDqStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 256);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    range[0] = 0x7fffffff;
    range[1] = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // elementwise threads: row 32 quarter + lane of the block, dims / keys half
  const int quarter = warp & 3;
  const int half = (warp - 2) >> 2;
  const int row = 32 * quarter + lane;
  int pos = -1, klo = 0, khi = 0;
  float lse = 0.0f, dsum = 0.0f;
  uint4 qv[8], dv[8];
  if (warp >= 2) {
    // rows past the routed count are absent (and may lie past this (b, g)'s packed rows)
    const bool present = R0 + row < cnt * p.r;
    const int64_t pr = packed_base(p, branch, b, g) + (present ? R0 + row : 0);
    int4 rec = make_int4(0, 0, 0, 0);
    if (present) {
      rec = p.rec[pr];
      pos = p.rpos[pr];
    }
    klo = rec.x;
    khi = rec.y;
    lse = __int_as_float(rec.z);
    dsum = __int_as_float(rec.w);
    if (half == 0 && khi > klo) {
      atomicMin(&range[0], klo);
      atomicMax(&range[1], khi);
    }
    // this thread's 64 dims of the row's Q and dO (in flight across the barrier)
    const uint4* qs = reinterpret_cast<const uint4*>(p.qp + pr * 128 + 64 * half);
    const uint4* ds = reinterpret_cast<const uint4*>(p.dop + pr * 128 + 64 * half);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      qv[j] = present ? __ldg(qs + j) : make_uint4(0, 0, 0, 0);
      dv[j] = present ? __ldg(ds + j) : make_uint4(0, 0, 0, 0);
    }
  }
  if (warp == 0) {
    __syncwarp();  // tcgen05.alloc is warp-collective: lane 0 comes from the set-up above
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int lo_u = range[0], hi_u = range[1];
  const int kfirst = lo_u < hi_u ? (lo_u / kDqKeys) * kDqKeys : 0;
  const int ntiles = lo_u < hi_u ? (hi_u - kfirst + kDqKeys - 1) / kDqKeys : 0;
  const uint32_t tm_q = tmem, tm_do = tmem + 64, tm_dq = tmem + 384;
  auto tm_s = [&](int t) { return tmem + 128 + 64 * (t & 1); };
  auto tm_dp = [&](int t) { return tmem + 256 + 64 * (t & 1); };

  if (warp == 0) {
    // ------------------------------------------------------------ K / V tiles
    if (lane == 0 && ntiles > 0) {
      tma_prefetch_desc(&p.k_map);
      tma_prefetch_desc(&p.v_map);
      int t = 0;
      for (; t < ntiles; ++t) {
        const int s = t % kDqStages;
        if (!mbar_wait(&empty[s], ((t / kDqStages) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], 2 * kDqKeyTile);
        uint8_t* dst = smem + DqTcSmem::stage + s * 2 * kDqKeyTile;
        const int key0 = kfirst + t * kDqKeys;
        tma_load_4d(dst, &p.k_map, &full[s], 0, g, key0, b);
        tma_load_4d(dst + kDqKeyTile / 2, &p.k_map, &full[s], 64, g, key0, b);
        tma_load_4d(dst + kDqKeyTile, &p.v_map, &full[s], 0, g, key0, b);
        tma_load_4d(dst + kDqKeyTile + kDqKeyTile / 2, &p.v_map, &full[s], 64, g, key0, b);
      }
      if (*abort_flag) {
        // let the loads already issued land before the CTA's shared memory is released
        for (int u = max(0, t - kDqStages); u < t; ++u) {
          volatile int dummy = 0;
          mbar_wait(&full[u % kDqStages], (u / kDqStages) & 1, &dummy);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 64, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, 128, false, true);
    auto product = [&](int t) {  // dQ += dS K of tile t (dS over the dP columns)
      const int s = t % kDqStages;
      const uint64_t k_mn = make_smem_desc_sw128(smem_u32(smem + DqTcSmem::stage + s * 2 * kDqKeyTile),
                                                 kDqKeyTile / 2, 1024);
#pragma unroll
      for (int c = 0; c < 2; ++c)  // keys 32 c .. 32 c + 31: BF16 pairs in columns 32 c .. 32 c + 15
        umma_ts_k32_warp(tm_dq, tm_dp(t) + 32 * c, k_mn + 2 * c * 128, idesc_o, (t > 0 || c > 0) ? 1u : 0u);
      tc_commit_warp(&empty[s]);
    };
    bool ok = ntiles == 0 || warp_wait(rows_full, 0, abort_flag);
    if (ok) tc_fence_after();
    for (int t = 0; t < ntiles && ok; ++t) {
      const int s = t % kDqStages;
      if (!warp_wait(&full[s], (t / kDqStages) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      // TMEM buffer t & 1 was last read by the product of tile t - 2, issued earlier
      const uint32_t ka = smem_u32(smem + DqTcSmem::stage + s * 2 * kDqKeyTile), va = ka + kDqKeyTile;
      umma_ts_k128_bhalf8k_warp(tm_s(t), tm_q, make_smem_desc_sw128(ka, 16, 1024), idesc_s);
      umma_ts_k128_bhalf8k_warp(tm_dp(t), tm_do, make_smem_desc_sw128(va, 16, 1024), idesc_s);
      tc_commit_warp(&s_full[t & 1]);
      if (t >= 1) {
        if (!warp_wait(&p_full[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        product(t - 1);
      }
    }
    if (ok && ntiles >= 1) {
      const int t = ntiles - 1;
      if (warp_wait(&p_full[t & 1], (t >> 1) & 1, abort_flag)) {
        tc_fence_after();
        product(t);
      }
    }
    // all MMAs complete before the epilogue reads (and before the CTA frees TMEM)
    tc_commit_warp(done);
  } else {
    // ------------------------------------------------------------ elementwise + epilogue
    const uint32_t lane_off = static_cast<uint32_t>(32 * quarter) << 16;
    {
      uint32_t r[32];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        r[4 * j] = qv[j].x;
        r[4 * j + 1] = qv[j].y;
        r[4 * j + 2] = qv[j].z;
        r[4 * j + 3] = qv[j].w;
      }
      tmem_st_x32(tm_q + lane_off + 32 * half, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        r[4 * j] = dv[j].x;
        r[4 * j + 1] = dv[j].y;
        r[4 * j + 2] = dv[j].z;
        r[4 * j + 3] = dv[j].w;
      }
      tmem_st_x32(tm_do + lane_off + 32 * half, r);
      tmem_st_wait();
    }
    tc_fence_before();
    mbar_arrive(rows_full);
    const float sl2 = p.scale_log2;
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int tb = t & 1;
      if (!warp_wait(&s_full[tb], (t >> 1) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[32], dr[32];
      tmem_ld_x32(tm_s(t) + lane_off + 32 * half, sr);
      tmem_ld_x32(tm_dp(t) + lane_off + 32 * half, dr);
      tmem_ld_wait();
      reg_fence32(sr);
      reg_fence32(dr);
      // legal keys of the row among this thread's 32: i in [i_lo, i_hi)
      const int key0 = kfirst + kDqKeys * t + 32 * half;
      const int i_lo = klo - key0, i_hi = khi - key0;
      uint32_t pk[16];
      if (__all_sync(0xffffffffu, i_lo <= 0 && i_hi >= 32)) {  // every entry of the warp legal
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float dsv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int i = 2 * j + e;
            dsv[e] = ex2_approx(__uint_as_float(sr[i]) * sl2 - lse) * (__uint_as_float(dr[i]) - dsum);
          }
          pk[j] = pack_bf16x2(dsv[0], dsv[1]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float dsv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int i = 2 * j + e;
            const bool legal = i >= i_lo && i < i_hi;
            const float pv = legal ? ex2_approx(__uint_as_float(sr[i]) * sl2 - lse) : 0.0f;
            dsv[e] = pv * (__uint_as_float(dr[i]) - dsum);
          }
          pk[j] = pack_bf16x2(dsv[0], dsv[1]);
        }
      }
      // over this thread's own, already read columns: 32 half .. 32 half + 15
      tmem_st_x16(tm_dp(t) + lane_off + 32 * half, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[tb]);
    }
    // epilogue: dQ (scaled) of this thread's row, dims 64 half .. 64 half + 63.
    // tcgen05.ld is warp-collective: every lane loads (the condition is warp
    // uniform), only the stores of absent rows are skipped.
    if (ok && ntiles > 0) ok = warp_wait(done, 0, abort_flag);
    tc_fence_after();
    const bool store = pos >= 0;
    const int64_t grow = (static_cast<int64_t>(b) * p.Sq + (store ? pos : 0)) * p.Hq + g * p.r + (R0 + row) % p.r;
    __nv_bfloat16* dst = p.dq + grow * 128 + 64 * half;
    const float sc = p.scale;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      uint32_t r[32];
      if (ntiles > 0 && ok) {
        tmem_ld_x32(tm_dq + lane_off + 64 * half + 32 * cc, r);
        tmem_ld_wait();
        reg_fence32(r);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
      if (store) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(r[8 * j]) * sc, __uint_as_float(r[8 * j + 1]) * sc);
          w.y = pack_bf16x2(__uint_as_float(r[8 * j + 2]) * sc, __uint_as_float(r[8 * j + 3]) * sc);
          w.z = pack_bf16x2(__uint_as_float(r[8 * j + 4]) * sc, __uint_as_float(r[8 * j + 5]) * sc);
          w.w = pack_bf16x2(__uint_as_float(r[8 * j + 6]) * sc, __uint_as_float(r[8 * j + 7]) * sc);
          *reinterpret_cast<uint4*>(dst + 32 * cc + 8 * j) = w;
        }
      }
    }
  }
  // teardown: the MMA warp's `done` commit covers every MMA it issued
  if (warp == 1) {
    volatile int dummy = 0;
    mbar_wait(done, 0, &dummy);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(p.status, kStatusTimeout);
}

}  // namespace

namespace {
size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
size_t packed_rows(int B, int Hq, int full_stride, int local_stride) {
  const size_t rows = static_cast<size_t>(B) * Hq * (static_cast<size_t>(full_stride) + local_stride);
  return rows > 0 ? rows : 1;
}
}  // namespace

size_t backward_workspace_bytes(int B, int Hq, int full_stride, int local_stride) {
  const size_t rows = packed_rows(B, Hq, full_stride, local_stride);
  return 256 + align256(rows * 16) + align256(rows * 4) + 2 * align256(rows * 256);
}

void bind_backward_workspace(BwdParams& p, void* workspace) {
  const size_t rows = packed_rows(p.B, p.Hq, p.idx_stride[0], p.idx_stride[1]);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  p.status = reinterpret_cast<int32_t*>(w);
  w += 256;
  p.rec = reinterpret_cast<int4*>(w);
  w += align256(rows * 16);
  p.rpos = reinterpret_cast<int32_t*>(w);
  w += align256(rows * 4);
  p.qp = reinterpret_cast<__nv_bfloat16*>(w);
  w += align256(rows * 256);
  p.dop = reinterpret_cast<__nv_bfloat16*>(w);
  p.pk_n0 = static_cast<int64_t>(p.B) * p.Hq * p.idx_stride[0];
  p.pk_rows = p.pk_n0 + static_cast<int64_t>(p.B) * p.Hq * p.idx_stride[1];
}

cudaError_t launch_backward(const BwdParams& params, int num_sms, cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDqTcSmemBytes);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(bwd_dkv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  if (params.pk_rows > 0) {
    const int64_t want = (params.pk_rows + 15) / 16;  // 16 rows per 256-thread block
    const int pack_blocks = static_cast<int>(want < 64LL * num_sms ? want : 64LL * num_sms);
    bwd_pack_kernel<<<pack_blocks, 256, 0, stream>>>(params);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 gq(params.nblk[0] + params.nblk[1], params.Hkv, params.B);
  if (gq.x > 0) bwd_dq_tc_kernel<<<gq, kDqThreads, kDqTcSmemBytes, stream>>>(params);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 gkv((params.Skv + kTcKeys - 1) / kTcKeys, params.Hkv, params.B);
  bwd_dkv_tc_kernel<<<gkv, kTcThreads, kTcSmemBytes, stream>>>(params);
  return cudaGetLastError();
}

}  // namespace swa
