// Switch Attention GQA prefill forward for B200 (sm_100a).
//
// One persistent kernel covers both branches of the reference's two launches
// (full causal: swiattn_gqa_prefill.py:8-214 with is_local=False; sliding window:
// is_local=True; varlen bounds: swiattn_gqa_prefill_varlen.py:33-249).
//
// Work unit: 256 query rows of one (branch, batch b, KV group g, head block hb)
// = PC routed positions x RP query heads of the group (RP = largest power of two
// dividing Hq/Hkv, at most 256; PC = 256 / RP), split into two 128-row tiles.
// Packing the heads that share a KV head into the MMA M dimension reads each K/V
// tile once per group instead of once per query head and narrows the position
// span of a tile, so the union key range wastes fewer masked entries.
//
// Roles (384 threads, one CTA per SM, persistent over a dynamic work counter):
//   warp 0      producer : TMA Q gather (one box per routed position) and the
//                          K/V tile ring (4 stages of 128 keys x 128 dims)
//   warp 1      MMA      : one thread issues tcgen05.mma
//                          S_i = Q_i K^T (SS, K-major) and O_i += P_i V (TS: P in TMEM,
//                          V MN-major), commits to mbarriers
//   warp 2      scheduler: fetches work units (atomic counter), publishes them
//                          through a shared-memory ring
//   warps 4-7   softmax 0: rows 0..127   (TMEM lane = row)
//   warps 8-11  softmax 1: rows 128..255
// TMEM (512 columns): S0 | S1 | O0 | O1, 128 FP32 columns each; P_i (BF16 pairs)
// overwrites the first 64 columns of S_i and is consumed by the next PV MMA.
//
// Numerics follow the reference: FP32 scores, log2-domain online softmax with
// scale_log2 = sm_scale * log2(e), running max initialised to -2^30 (scaled),
// P rounded to BF16 before P V, the row sum accumulated from the unrounded FP32
// P, O = acc / l and LSE = log2(l) + m.  The running max is only raised (and O
// rescaled) when it grows by more than 8 (a factor 256), which leaves the final
// O and LSE mathematically unchanged while removing most O rescales.
#include "sm100.cuh"
#include "swattn_internal.h"

namespace swa {

namespace {

constexpr int kThreads = 384;
constexpr int kBK = 128;            // keys per K/V tile
constexpr int kStages = 4;          // K/V ring depth (each stage: one K or one V tile)
constexpr int kSchedSlots = 4;      // work-unit ring depth
constexpr uint32_t kTileBytes = 128 * 128 * 2;   // 32 KB: a 128x128 BF16 tile (2 swizzled halves)
constexpr uint32_t kHalfBytes = 128 * 64 * 2;    // 16 KB: 128 rows x 64 columns
constexpr float kRescaleThreshold = 8.0f;

struct Unit {
  int valid;    // 0 = no more work
  int branch;   // 0 = full, 1 = local
  int b, g, hb, pb;
  int count;    // routed rows of this (branch, b)
  int j0, n;    // first key tile and number of key tiles
  int pad[7];
};

struct SmemLayout {
  // offsets (bytes) from the 1024-aligned dynamic shared memory base
  static constexpr uint32_t q0 = 0;
  static constexpr uint32_t q1 = kTileBytes;
  static constexpr uint32_t kv = 2 * kTileBytes;
  static constexpr uint32_t bars = kv + kStages * kTileBytes;
  // barrier indices
  static constexpr int b_sched_full = 0;
  static constexpr int b_sched_empty = b_sched_full + kSchedSlots;
  static constexpr int b_q_full = b_sched_empty + kSchedSlots;
  static constexpr int b_q_empty = b_q_full + 2;
  static constexpr int b_kv_full = b_q_empty + 2;
  static constexpr int b_kv_empty = b_kv_full + kStages;
  static constexpr int b_s_full = b_kv_empty + kStages;
  static constexpr int b_p_full = b_s_full + 2;
  static constexpr int b_o_full = b_p_full + 2;
  static constexpr int b_o_empty = b_o_full + 2;
  static constexpr int b_drain = b_o_empty + 2;
  static constexpr int n_bars = b_drain + 1;
  static constexpr uint32_t units = bars + ((n_bars * 8 + 63) / 64) * 64;
  static constexpr uint32_t misc = units + kSchedSlots * sizeof(Unit);
  static constexpr uint32_t total = misc + 64;
};

constexpr uint32_t kSmemBytes = SmemLayout::total + 1024;  // + alignment slack

struct RowBounds {
  int lo, hi;
};

__device__ __forceinline__ RowBounds row_bounds(const PrefillParams& p, int branch, int qpos) {
  RowBounds r;
  if (p.ends != nullptr) {
    r.lo = max(p.starts[branch][qpos], 0);
    r.hi = min(p.ends[qpos], p.Skv);
  } else {
    r.lo = branch ? max(qpos - p.window + 1, 0) : 0;
    r.hi = min(qpos + 1, p.Skv);
  }
  return r;
}

__device__ __forceinline__ int branch_count(const PrefillParams& p, int branch, int b) {
  return p.counts != nullptr ? p.counts[branch * p.B + b] : p.count_scalar[branch];
}

__device__ __forceinline__ int load_pos(const PrefillParams& p, int branch, int b, int slot) {
  return p.idx[branch][static_cast<int64_t>(b) * p.idx_stride[branch] + slot];
}

// Decode work item `it` into a unit; returns false for an empty item.
__device__ bool decode_item(const PrefillParams& p, int it, int nf, int maxnpb0, int maxnpb1, Unit& u) {
  const int per_level = p.n_bg * p.nhb;
  int branch, pb, rem;
  if (it < nf) {
    branch = 0;
    pb = maxnpb0 - 1 - it / per_level;  // longest full-causal units first
    rem = it % per_level;
  } else {
    it -= nf;
    branch = 1;
    pb = maxnpb1 - 1 - it / per_level;
    rem = it % per_level;
  }
  const int bgi = rem / p.nhb;
  const int hb = rem % p.nhb;
  const int bg = p.bg_list != nullptr ? p.bg_list[bgi] : bgi;
  const int b = bg / p.Hkv;
  const int g = bg % p.Hkv;
  const int cnt = min(branch_count(p, branch, b), p.idx_cap[branch]);
  const int first_slot = pb * p.pc;
  if (first_slot >= cnt) return false;
  const int last_slot = min(first_slot + p.pc, cnt) - 1;
  const int fpos = min(max(load_pos(p, branch, b, first_slot), 0), p.Sq - 1);
  const int lpos = min(max(load_pos(p, branch, b, last_slot), 0), p.Sq - 1);
  int lo, hi;
  if (p.ends != nullptr) {
    lo = max(p.starts[branch][fpos], 0);
    hi = min(p.ends[lpos], p.Skv);
  } else {
    lo = branch ? max(fpos - p.window + 1, 0) : 0;
    hi = min(lpos + 1, p.Skv);
  }
  const int j0 = lo / kBK;
  const int j1 = (hi + kBK - 1) / kBK;
  u.valid = 1;
  u.branch = branch;
  u.b = b;
  u.g = g;
  u.hb = hb;
  u.pb = pb;
  u.count = cnt;
  u.j0 = j0;
  u.n = max(j1 - j0, 0);
  return true;
}

__device__ __forceinline__ void read_unit(const volatile Unit* src, Unit& u) {
  u.valid = src->valid;
  u.branch = src->branch;
  u.b = src->b;
  u.g = src->g;
  u.hb = src->hb;
  u.pb = src->pb;
  u.count = src->count;
  u.j0 = src->j0;
  u.n = src->n;
}

__global__ void __launch_bounds__(kThreads, 1) switch_prefill_kernel(const __grid_constant__ PrefillParams p) {
  if (p.gate != nullptr && *p.gate != 0) return;  // index validation failed: write nothing

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemLayout::bars);
  Unit* units = reinterpret_cast<Unit*>(smem + SmemLayout::units);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + SmemLayout::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + SmemLayout::misc + 4);

  uint64_t* sched_full = bars + SmemLayout::b_sched_full;
  uint64_t* sched_empty = bars + SmemLayout::b_sched_empty;
  uint64_t* q_full = bars + SmemLayout::b_q_full;
  uint64_t* q_empty = bars + SmemLayout::b_q_empty;
  uint64_t* kv_full = bars + SmemLayout::b_kv_full;
  uint64_t* kv_empty = bars + SmemLayout::b_kv_empty;
  uint64_t* s_full = bars + SmemLayout::b_s_full;
  uint64_t* p_full = bars + SmemLayout::b_p_full;
  uint64_t* o_full = bars + SmemLayout::b_o_full;
  uint64_t* o_empty = bars + SmemLayout::b_o_empty;
  uint64_t* drain = bars + SmemLayout::b_drain;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSchedSlots; ++s) {
      mbar_init(&sched_full[s], 1);
      mbar_init(&sched_empty[s], 1 + 1 + 256);  // producer lane 0, MMA lane 0, 256 softmax threads
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 128);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.q_map);
    tma_prefetch_desc(&p.k_map);
    tma_prefetch_desc(&p.v_map);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 2) {
    // ------------------------------------------------------------------ scheduler
    if (lane == 0) {
      int maxnpb0 = 0, maxnpb1 = 0;
      for (int b = 0; b < p.B; ++b) {
        maxnpb0 = max(maxnpb0, (min(branch_count(p, 0, b), p.idx_cap[0]) + p.pc - 1) / p.pc);
        maxnpb1 = max(maxnpb1, (min(branch_count(p, 1, b), p.idx_cap[1]) + p.pc - 1) / p.pc);
      }
      const int per_level = p.n_bg * p.nhb;
      const int nf = maxnpb0 * per_level;
      const int total = nf + maxnpb1 * per_level;
      for (int k = 0;; ++k) {
        const int slot = k % kSchedSlots;
        if (!mbar_wait(&sched_empty[slot], ((k / kSchedSlots) & 1) ^ 1, abort_flag)) break;
        Unit u;
        u.valid = 0;
        while (true) {
          const int it = atomicAdd(p.counter, 1);
          if (it >= total) break;
          if (decode_item(p, it, nf, maxnpb0, maxnpb1, u)) break;
        }
        volatile Unit* dst = &units[slot];
        dst->valid = u.valid;
        dst->branch = u.branch;
        dst->b = u.b;
        dst->g = u.g;
        dst->hb = u.hb;
        dst->pb = u.pb;
        dst->count = u.count;
        dst->j0 = u.j0;
        dst->n = u.n;
        mbar_arrive(&sched_full[slot]);
        if (!u.valid) break;
      }
    }
  } else if (warp == 0) {
    // ------------------------------------------------------------------ producer
    uint32_t kv_it = 0;
    uint32_t q_use[2] = {0, 0};
    const int r = p.Hq / p.Hkv;
    const int boxes = 128 / p.boxh;  // boxes per tile per 64-column half
    for (int k = 0;; ++k) {
      const int slot = k % kSchedSlots;
      if (!mbar_wait(&sched_full[slot], (k / kSchedSlots) & 1, abort_flag)) break;
      Unit u;
      read_unit(&units[slot], u);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sched_empty[slot]);
      if (!u.valid) break;
      if (u.n == 0) continue;
      bool ok = true;
      for (int i = 0; i < 2 && ok; ++i) {
        if (!mbar_wait(&q_empty[i], (q_use[i] & 1) ^ 1, abort_flag)) { ok = false; break; }
        ++q_use[i];
        if (lane == 0) mbar_arrive_expect_tx(&q_full[i], kTileBytes);
        __syncwarp();
        uint8_t* qdst = smem + (i == 0 ? SmemLayout::q0 : SmemLayout::q1);
        for (int t = lane; t < 2 * boxes; t += 32) {
          const int half = t & 1;
          const int bx = t >> 1;
          const int row0 = 128 * i + bx * p.boxh;          // first unit row of this box
          const int slot_in_unit = row0 / p.rp;
          const int hoff = row0 % p.rp;
          const int slot_abs = min(u.pb * p.pc + slot_in_unit, u.count - 1);
          const int pos = min(max(load_pos(p, u.branch, u.b, slot_abs), 0), p.Sq - 1);
          const int row = (u.b * p.Sq + pos) * p.Hq + u.g * r + u.hb * p.rp + hoff;
          tma_load_2d(qdst + half * kHalfBytes + bx * p.boxh * 128, &p.q_map, &q_full[i], half * 64, row);
        }
      }
      if (!ok) break;
      for (int j = 0; j < u.n && ok; ++j) {
        const int key0 = (u.j0 + j) * kBK;
        for (int kv = 0; kv < 2; ++kv) {
          const uint32_t s = kv_it % kStages;
          if (!mbar_wait(&kv_empty[s], ((kv_it / kStages) & 1) ^ 1, abort_flag)) { ok = false; break; }
          if (lane == 0) {
            mbar_arrive_expect_tx(&kv_full[s], kTileBytes);
            uint8_t* dst = smem + SmemLayout::kv + s * kTileBytes;
            const CUtensorMap* map = kv == 0 ? &p.k_map : &p.v_map;
            tma_load_4d(dst, map, &kv_full[s], 0, u.g, key0, u.b);
            tma_load_4d(dst + kHalfBytes, map, &kv_full[s], 64, u.g, key0, u.b);
          }
          __syncwarp();
          ++kv_it;
        }
      }
      if (!ok) break;
    }
    if (*abort_flag) {
      // Let every load already issued land before the CTA releases its memory.
      for (uint32_t s = 0; s < kStages && s < kv_it; ++s) {
        const uint32_t last = kv_it - 1 - ((kv_it - 1 - s) % kStages);
        volatile int dummy = 0;
        mbar_wait(&kv_full[last % kStages], (last / kStages) & 1, &dummy);
      }
      for (int i = 0; i < 2; ++i) {
        if (q_use[i] > 0) {
          volatile int dummy = 0;
          mbar_wait(&q_full[i], (q_use[i] - 1) & 1, &dummy);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, 128, false, true);
    const uint32_t q_addr[2] = {smem_u32(smem + SmemLayout::q0), smem_u32(smem + SmemLayout::q1)};
    const uint32_t kv_addr = smem_u32(smem + SmemLayout::kv);
    const uint32_t tm_s[2] = {tmem + 0, tmem + 128};
    const uint32_t tm_o[2] = {tmem + 256, tmem + 384};
    uint32_t kv_it = 0, q_use[2] = {0, 0}, p_use[2] = {0, 0}, o_use = 0;
    bool ok = true;
    auto issue_s = [&](int i, uint32_t kstage) {
      const uint32_t kb = kv_addr + kstage * kTileBytes;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
        umma_ss(tm_s[i], make_smem_desc_sw128(q_addr[i] + off, 16, 1024), make_smem_desc_sw128(kb + off, 16, 1024),
                idesc_s, kk > 0 ? 1u : 0u);
      }
    };
    auto issue_pv = [&](int i, uint32_t vstage, bool accumulate) {
      const uint32_t vb = kv_addr + vstage * kTileBytes;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        umma_ts(tm_o[i], tm_s[i] + kk * 8, make_smem_desc_sw128(vb + kk * 2048, kHalfBytes, 1024), idesc_o,
                (accumulate || kk > 0) ? 1u : 0u);
      }
    };
    for (int k = 0; ok; ++k) {
      const int slot = k % kSchedSlots;
      if (!mbar_wait(&sched_full[slot], (k / kSchedSlots) & 1, abort_flag)) break;
      Unit u;
      read_unit(&units[slot], u);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sched_empty[slot]);
      if (!u.valid) break;
      if (u.n == 0) continue;
      if (lane == 0) {
        // prologue: S_0(0), S_1(0)
        uint32_t ks = kv_it % kStages;
        ok = ok && mbar_wait(&q_full[0], q_use[0] & 1, abort_flag);
        ok = ok && mbar_wait(&kv_full[ks], (kv_it / kStages) & 1, abort_flag);
        if (ok) {
          ++q_use[0];
          tc_fence_after();
          issue_s(0, ks);
          tc_commit(&s_full[0]);
        }
        ok = ok && mbar_wait(&q_full[1], q_use[1] & 1, abort_flag);
        if (ok) {
          ++q_use[1];
          tc_fence_after();
          issue_s(1, ks);
          tc_commit(&s_full[1]);
          if (u.n == 1) {
            tc_commit(&q_empty[0]);
            tc_commit(&q_empty[1]);
          }
          tc_commit(&kv_empty[ks]);
          ++kv_it;
        }
        for (int j = 0; j < u.n && ok; ++j) {
          const uint32_t vs = kv_it % kStages;
          ok = ok && mbar_wait(&kv_full[vs], (kv_it / kStages) & 1, abort_flag);
          ++kv_it;
          ok = ok && mbar_wait(&p_full[0], p_use[0] & 1, abort_flag);
          ++p_use[0];
          if (j == 0) ok = ok && mbar_wait(&o_empty[0], (o_use & 1) ^ 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
          issue_pv(0, vs, j > 0);
          uint32_t ks_next = 0;
          const bool more = j + 1 < u.n;
          if (more) {
            ks_next = kv_it % kStages;
            ok = ok && mbar_wait(&kv_full[ks_next], (kv_it / kStages) & 1, abort_flag);
            ++kv_it;
            if (!ok) break;
            issue_s(0, ks_next);
            tc_commit(&s_full[0]);
            if (j + 2 == u.n) tc_commit(&q_empty[0]);
          } else {
            tc_commit(&o_full[0]);
          }
          ok = ok && mbar_wait(&p_full[1], p_use[1] & 1, abort_flag);
          ++p_use[1];
          if (j == 0) ok = ok && mbar_wait(&o_empty[1], (o_use & 1) ^ 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
          issue_pv(1, vs, j > 0);
          tc_commit(&kv_empty[vs]);
          if (more) {
            issue_s(1, ks_next);
            tc_commit(&s_full[1]);
            if (j + 2 == u.n) tc_commit(&q_empty[1]);
            tc_commit(&kv_empty[ks_next]);
          } else {
            tc_commit(&o_full[1]);
          }
        }
        ++o_use;
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
    if (lane == 0) {
      // drain: wait until every MMA issued by this thread has completed
      tc_commit(drain);
      volatile int dummy = 0;
      mbar_wait(drain, 0, &dummy);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax / epilogue
    const int tile = (warp - 4) >> 2;            // 0 or 1
    const int t = threadIdx.x - 128 * (1 + tile);  // row within the tile = TMEM lane
    const int lane_base = (warp & 3) * 32;
    const uint32_t tm_s = tmem + 128 * tile + (static_cast<uint32_t>(lane_base) << 16);
    const uint32_t tm_o = tmem + 256 + 128 * tile + (static_cast<uint32_t>(lane_base) << 16);
    const int R = 128 * tile + t;                  // row within the unit
    const int slot_in_unit = R / p.rp;
    const int head_in_group_off = R % p.rp;
    const int r = p.Hq / p.Hkv;
    const float sl2 = p.scale_log2;
    const float m_init = -1073741824.0f * sl2;     // reference initial row max (-2^30), scaled
    uint32_t s_use = 0, o_use = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int slot = k % kSchedSlots;
      if (!mbar_wait(&sched_full[slot], (k / kSchedSlots) & 1, abort_flag)) break;
      Unit u;
      read_unit(&units[slot], u);
      mbar_arrive(&sched_empty[slot]);
      if (!u.valid) break;
      const int slot_abs = u.pb * p.pc + slot_in_unit;
      int qpos = -1;
      if (slot_abs < u.count) qpos = load_pos(p, u.branch, u.b, slot_abs);
      const bool valid_row = qpos >= 0 && qpos < p.Sq;
      RowBounds rb = {0, 0};
      if (valid_row) rb = row_bounds(p, u.branch, qpos);
      const int head = u.g * r + u.hb * p.rp + head_in_group_off;
      const int64_t orow = valid_row ? (static_cast<int64_t>(u.b) * p.Sq + qpos) * p.Hq + head : 0;
      if (u.n == 0) {
        if (valid_row) {
          const uint32_t nan_pair = 0x7FC07FC0u;
          uint4* dst = reinterpret_cast<uint4*>(p.out + orow * 128);
#pragma unroll
          for (int c = 0; c < 16; ++c) dst[c] = make_uint4(nan_pair, nan_pair, nan_pair, nan_pair);
          p.lse[orow] = -INFINITY;
        }
        continue;
      }
      float m = m_init;
      float l = 0.0f;
      for (int j = 0; j < u.n; ++j) {
        if (!mbar_wait(&s_full[tile], s_use & 1, abort_flag)) { ok = false; break; }
        ++s_use;
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld_x32(tm_s + 0, sr + 0);
        tmem_ld_x32(tm_s + 32, sr + 32);
        tmem_ld_x32(tm_s + 64, sr + 64);
        tmem_ld_x32(tm_s + 96, sr + 96);
        tmem_ld_wait();
        reg_fence32(sr + 0);
        reg_fence32(sr + 32);
        reg_fence32(sr + 64);
        reg_fence32(sr + 96);
        float* s = reinterpret_cast<float*>(sr);
        const int k0 = (u.j0 + j) * kBK;
        if (!(rb.lo <= k0 && k0 + kBK <= rb.hi)) {
#pragma unroll
          for (int e = 0; e < 128; ++e) {
            const int key = k0 + e;
            if (key < rb.lo || key >= rb.hi) s[e] = -INFINITY;
          }
        }
        float mx = s[0];
#pragma unroll
        for (int e = 1; e < 128; ++e) mx = fmaxf(mx, s[e]);
        const float m_tile = mx * sl2;
        bool rescale = false;
        float alpha = 1.0f;
        if (l == 0.0f) {
          m = fmaxf(m, m_tile);
        } else if (m_tile > m + kRescaleThreshold) {
          alpha = ex2_approx(m - m_tile);
          l *= alpha;
          m = m_tile;
          rescale = true;
        }
        const float neg_m = -m;
        float sum = 0.0f;
        uint32_t pk[64];
#pragma unroll
        for (int e = 0; e < 128; e += 2) {
          const float p0 = ex2_approx(fmaf(s[e], sl2, neg_m));
          const float p1 = ex2_approx(fmaf(s[e + 1], sl2, neg_m));
          sum += p0 + p1;
          pk[e >> 1] = pack_bf16x2(p0, p1);
        }
        l += sum;
        tmem_st_x32(tm_s + 0, pk);
        tmem_st_x32(tm_s + 32, pk + 32);
        if (__any_sync(0xffffffffu, rescale)) {
          // O_tile (PV of earlier key tiles, all complete) *= alpha for this row
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t orr[32];
            tmem_ld_x32(tm_o + 32 * c, orr);
            tmem_ld_wait();
            reg_fence32(orr);
#pragma unroll
            for (int e = 0; e < 32; ++e) orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
            tmem_st_x32(tm_o + 32 * c, orr);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[tile]);
      }
      if (!ok) break;
      // epilogue: O / l -> BF16 at the row's original position, LSE in log2 units
      if (!mbar_wait(&o_full[tile], o_use & 1, abort_flag)) { ok = false; break; }
      ++o_use;
      tc_fence_after();
      const float inv_l = 1.0f / l;
      uint4 packed[16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t orr[32];
        tmem_ld_x32(tm_o + 32 * c, orr);
        tmem_ld_wait();
        reg_fence32(orr);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(orr[q4 * 8 + 0]) * inv_l, __uint_as_float(orr[q4 * 8 + 1]) * inv_l);
          w.y = pack_bf16x2(__uint_as_float(orr[q4 * 8 + 2]) * inv_l, __uint_as_float(orr[q4 * 8 + 3]) * inv_l);
          w.z = pack_bf16x2(__uint_as_float(orr[q4 * 8 + 4]) * inv_l, __uint_as_float(orr[q4 * 8 + 5]) * inv_l);
          w.w = pack_bf16x2(__uint_as_float(orr[q4 * 8 + 6]) * inv_l, __uint_as_float(orr[q4 * 8 + 7]) * inv_l);
          packed[c * 4 + q4] = w;
        }
      }
      tc_fence_before();
      mbar_arrive(&o_empty[tile]);
      if (valid_row) {
        uint4* dst = reinterpret_cast<uint4*>(p.out + orow * 128);
#pragma unroll
        for (int c = 0; c < 16; ++c) dst[c] = packed[c];
        p.lse[orow] = lg2_approx(l) + m;
      }
    }
  }

  // ------------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(p.status, kStatusTimeout);
}

}  // namespace

cudaError_t launch_prefill(const PrefillParams& params, int num_sms, cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(switch_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  switch_prefill_kernel<<<num_sms, kThreads, kSmemBytes, stream>>>(params);
  return cudaGetLastError();
}

uint32_t prefill_smem_bytes() { return kSmemBytes; }

}  // namespace swa
