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
// Roles (576 threads, one CTA per SM, persistent over a dynamic work counter):
//   warp 0      producer : takes work units from the global counter (the next one
//                          while the current unit's last key tiles load) and
//                          publishes them through a shared-memory ring;
//                          TMA Q gather (boxes of consecutive routed positions, see
//                          q_tile_boxes) and the K/V tile ring (5 entries of 128
//                          keys x 128 dims, one TMA box each, K and V alternating);
//                          K/V loads evict-last in L2, Q loads and O stores evict-first
//   warp 1      MMA      : one elected lane issues tcgen05.mma in groups of eight
//                          (S) or two (P V chunk) instructions:
//                          S_i = Q_i K^T (SS, K-major) and O_i += P_i V (TS: P in TMEM,
//                          V MN-major), commits to mbarriers.  Its issue order is one
//                          continuous stream over key steps: PV_0(j), S_0(j+1),
//                          PV_1(j), S_1(j+1); at a unit's last step both P V groups
//                          go first, then the next unit's S MMAs.
//   warps 2-17  softmax  : tile = (warp - 2) / 8 (rows 0..127 or 128..255 of the
//                          unit, TMEM lane = row); the two warps of a tile on one
//                          TMEM lane quarter take its lanes 0-15 and 16-31, and within
//                          a warp threads l and l + 16 share a row (16-lane TMEM
//                          loads: keys [0, 32) + [64, 96) and [32, 64) + [96, 128) of
//                          each key tile), exchanging row max and row sum by warp
//                          shuffle; then the O/LSE epilogue of the tile.
// TMEM (512 columns): S0 | S1 | O0 | O1, 128 FP32 columns each; P_i (BF16 pairs) of
// keys [64 c, 64 c + 64) overwrites columns 32 c .. 32 c + 31 of S_i (scores the
// threads already hold) and is consumed by the next PV MMA.  P is published in two
// chunks (c = 0, 1).
// Key tiles of a unit start at the 64-aligned key at or below its first legal key.
//
// Numerics follow the reference: FP32 scores, log2-domain online softmax with
// scale_log2 = sm_scale * log2(e), running max initialised to -2^30 (scaled),
// P rounded to BF16 before P V, the row sum accumulated from the unrounded FP32
// P, O = acc / l and LSE = log2(l) + m.  The running max is only raised (and O
// rescaled) when it grows by more than 8 (a factor 256), which leaves the final
// O and LSE mathematically unchanged while removing most O rescales.  One pair of
// exponentials in four is evaluated on the FMA pipe (exp2_poly_pair) instead of
// the MUFU unit, which otherwise bounds the softmax rate.
#include <algorithm>
#include <cmath>

#include "sm100.cuh"
#include "swattn_internal.h"

namespace swa {

namespace {

constexpr int kThreads = 576;
constexpr int kBK = 128;            // keys per K/V tile
constexpr int kStages = 5;          // K/V ring depth (each stage: one K or one V tile)
constexpr int kSchedSlots = 4;      // work-unit ring depth
constexpr int kFetchAheadTiles = 2; // the next unit is claimed while the last 3 key tiles load
constexpr uint32_t kTileBytes = 128 * 128 * 2;   // 32 KB: a 128x128 BF16 tile (2 swizzled halves)
constexpr uint32_t kHalfBytes = 128 * 64 * 2;    // 16 KB: 128 rows x 64 columns
constexpr float kRescaleThreshold = 8.0f;
// L2 use: K/V tiles are read by every unit of their (b, g) group, Q rows and O rows
// are touched once.  The K/V loads carry an evict-last L2 policy, the Q loads and
// O stores evict-first, so the streams of Q and O do not push the groups' K/V
// prefixes out of L2 (config 3: DRAM traffic per launch 5.72 -> 4.34 GB; the Q L2
// prefetch one unit ahead that this replaced added 1.1 GB of re-reads).

struct Unit {
  int valid;    // 0 = no more work
  int branch;   // 0 = full, 1 = local
  int b, g, hb, pb;
  int count;    // routed rows of this (branch, b)
  int j0, n;    // first key (a multiple of 64) / 64, and number of 128-key tiles from there
  int part;     // key-split piece: its scratch slot (-1: the unit is not split)
  int pad[6];
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
  static constexpr int b_p_chunk = b_s_full + 2;   // [tile][key chunk]
  static constexpr int b_o_full = b_p_chunk + 4;
  static constexpr int b_o_empty = b_o_full + 2;
  static constexpr int b_drain = b_o_empty + 2;
  static constexpr int n_bars = b_drain + 1;
  static constexpr uint32_t units = bars + ((n_bars * 8 + 63) / 64) * 64;
  static constexpr uint32_t misc = units + kSchedSlots * sizeof(Unit);
  static constexpr uint32_t total = misc + 64;
};

constexpr uint32_t kSmemBytes = SmemLayout::total + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "dynamic shared memory above the 227 KB a CTA may use");

struct RowBounds {
  int lo, hi;
};

// Optional cycle-level event trace of CTA 0 (compiled only with -DSWA_TRACE): each
// recorder (MMA issuer, softmax warpgroup 0, softmax warpgroup 1, producer) appends
// (event id, key step, clock64) records to its own region of g_swa_trace.
#ifdef SWA_TRACE
__device__ unsigned long long* g_swa_trace = nullptr;
constexpr int kTraceCap = 8192;
struct Tracer {
  unsigned long long* buf;
  int n;
  __device__ explicit Tracer(int recorder)
      : buf(blockIdx.x == 0 && recorder >= 0 && g_swa_trace != nullptr
                ? g_swa_trace + static_cast<size_t>(recorder) * 2 * kTraceCap
                : nullptr),
        n(0) {}
  __device__ __forceinline__ void ev(int id, int step) {
    if (buf != nullptr && n < kTraceCap) {
      buf[2 * n] = (static_cast<unsigned long long>(id) << 32) | static_cast<unsigned>(step);
      buf[2 * n + 1] = clock64();
      ++n;
    }
  }
};
#else
struct Tracer {
  __device__ explicit Tracer(int) {}
  __device__ __forceinline__ void ev(int, int) {}
};
#endif

// Optional per-CTA duration in SM clock cycles (compiled only with -DSWA_CYCLES),
// for comparing kernel variants independently of the clock frequency.
#ifdef SWA_CYCLES
__device__ unsigned long long g_swa_cycles[1024];
#endif

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
  return p.counts != nullptr ? p.counts[branch * p.cs_branch + b * p.cs_batch] : p.count_scalar[branch];
}

__device__ __forceinline__ int load_pos(const PrefillParams& p, int branch, int b, int slot) {
  return p.idx[branch][static_cast<int64_t>(b) * p.idx_stride[branch] + slot];
}

// Row of (batch b of this launch, position, head of the launch) in the replicated
// row-major outputs: batch b is global unit unit_gid[b] = b_g * rep_hkv + g_g, and
// the launch's Hq heads are that unit's KV group (launches over unit-major inputs,
// Hkv == 1).
__device__ __forceinline__ int64_t replica_row(const PrefillParams& p, int b, int qpos, int head) {
  const int gid = p.unit_gid[b];
  const int bg = gid / p.rep_hkv, gg = gid - bg * p.rep_hkv;
  const int hq_g = p.rep_hkv * p.Hq;
  return (static_cast<int64_t>(bg) * p.Sq + qpos) * hq_g + static_cast<int64_t>(gg) * p.Hq + head;
}

// Decode work item `it` into a unit; returns false for an empty item.
//
// Items are ordered (b, g)-major: all full-branch units of one (batch, KV group),
// longest first, then its local-branch units (last positions first), then the
// next group.  The CTAs running at one time then stream the K/V of a few groups
// (16 MB each at S = 32K), which stays in L2 while every unit of those groups,
// full and local, reads it.  Ordered by length across all groups, the full units
// streamed the prefixes of every group at once; with every local unit after every
// full unit, the local units read each group's K/V from DRAM a second time
// (config 3, B = 4: 2x the K/V bytes).  The tail stays short: the local units of
// the last kTailGroups groups (all about W keys) come after every full unit,
// position-block-major over those groups, and fill the CTAs while the last long
// full units finish (config 3: with 4 such groups a launch took 4 % more cycles
// than with 8; each group kept for the tail reads its K/V a second time).
constexpr int kTailGroups = 8;

// Key tiles of the unit of (branch, b) whose routed slots start at first_slot
// (< cnt): the union of its rows' key ranges from the first and last routed row,
// in 128-key tiles from the 64-aligned key at or below the first legal key.
__device__ __forceinline__ void unit_tiles(const PrefillParams& p, int branch, int b, int first_slot, int cnt,
                                           int& j0, int& n) {
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
  // key tiles start at the 64-aligned key at or below lo (a 128-key grid would
  // waste up to 64 more masked keys per row)
  j0 = lo / 64;
  n = max((hi - j0 * 64 + kBK - 1) / kBK, 0);
}

// Pieces of a full-branch unit of n key tiles under a key split: np pieces of
// len tiles (the last one shorter), of which the first `used` start below n.
__device__ __forceinline__ void split_pieces(const PrefillParams& p, int n, int& np, int& len, int& used) {
  np = (p.split_tiles > 0 && n > p.split_tiles) ? (n + p.split_tiles - 1) / p.split_tiles : 1;
  len = (n + np - 1) / np;
  used = len > 0 ? (n + len - 1) / len : 1;
}

template <bool kSplit>
__device__ bool decode_item(const PrefillParams& p, int it, int maxnpb0, int maxnpb1, Unit& u) {
  const int P = kSplit ? p.pieces : 1;   // work items per full-branch unit (1: no key split)
  const int per0 = maxnpb0 * p.nhb * P;  // full-branch items of one group
  const int per1 = maxnpb1 * p.nhb;      // local-branch items of one group
  const int n_early = max(p.n_bg - kTailGroups, 0);
  const int early_items = n_early * (per0 + per1);
  int branch, pb, rem, piece = 0;
  if (it < early_items) {
    const int grp = it / (per0 + per1);
    int w = it - grp * (per0 + per1);
    if (w < per0) {
      branch = 0;
      pb = maxnpb0 - 1 - w / (p.nhb * P);  // longest full-causal units of the group first
      piece = w % P;
      w /= P;
    } else {
      w -= per0;
      branch = 1;
      pb = maxnpb1 - 1 - w / p.nhb;
    }
    rem = grp * p.nhb + w % p.nhb;
  } else {
    it -= early_items;
    const int n_late = p.n_bg - n_early;
    if (it < n_late * per0) {
      branch = 0;
      const int grp = n_early + it / per0;
      const int w = it % per0;
      pb = maxnpb0 - 1 - w / (p.nhb * P);
      piece = w % P;
      rem = grp * p.nhb + (w / P) % p.nhb;
    } else {
      it -= n_late * per0;
      branch = 1;
      pb = maxnpb1 - 1 - it / (n_late * p.nhb);
      rem = n_early * p.nhb + it % (n_late * p.nhb);
    }
  }
  const int bgi = rem / p.nhb;
  const int hb = rem % p.nhb;
  const int bg = p.bg_list != nullptr ? p.bg_list[bgi] : bgi;
  const int b = bg / p.Hkv;
  const int g = bg % p.Hkv;
  const int cnt = min(branch_count(p, branch, b), p.idx_cap[branch]);
  const int first_slot = pb * p.pc;
  if (first_slot >= cnt) return false;
  int j0, n;
  unit_tiles(p, branch, b, first_slot, cnt, j0, n);
  int part = -1;
  if (kSplit && branch == 0 && P > 1) {
    int np, len, used;
    split_pieces(p, n, np, len, used);
    // the scratch holds the split_pb_cap longest units of each (unit, head block):
    // rank rr from the end of the branch's position blocks; a longer-ranked unit
    // runs whole
    const int rr = (cnt + p.pc - 1) / p.pc - 1 - pb;
    if (rr >= p.split_pb_cap) {
      np = 1;
      used = 1;
    }
    if (piece >= used) return false;  // no such piece: an empty item
    if (np > 1) {
      j0 += 2 * piece * len;          // j0 counts 64-key steps, a tile is two
      n = min(len, n - piece * len);
      part = ((bgi * p.nhb + hb) * p.split_pb_cap + rr) * P + piece;
    }
  }
  u.valid = 1;
  u.branch = branch;
  u.b = b;
  u.g = g;
  u.hb = hb;
  u.pb = pb;
  u.count = cnt;
  u.j0 = j0;
  u.n = n;
  u.part = part;
  return true;
}

template <bool kSplit>
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
  u.part = kSplit ? src->part : -1;
}

// TMA boxes of Q tile i (rows 128 i .. 128 i + 127) of unit u, issued by the
// producer warp's lanes into `qdst`, completing on `bar` (evict-first L2 policy:
// every Q row is read once).  With rp <= 64 a tile holds spt = 128 / rp routed
// positions (slots); each slot s is covered by the largest aligned power-of-two
// block of slots containing it whose positions are consecutive, and such a block
// of 2^L slots is one box of 2^L positions x rp heads (3-D map q_runs[L - 1]), or
// of rp rows (2-D map) for a single slot.  Blocks of consecutive positions contain
// sub-blocks of consecutive positions, so these maximal blocks partition the slots
// and every row is loaded exactly once.
__device__ __forceinline__ void q_tile_boxes(const PrefillParams& p, const Unit& u, int i, int lane, uint8_t* qdst,
                                             uint64_t* bar) {
  const int head0 = u.g * (p.Hq / p.Hkv) + u.hb * p.rp;
  const uint64_t pol = l2_policy_evict_first();
  if (p.rp > 64) {
    // at most one position per tile: boxes of boxh rows (rp = 128: one box per half;
    // rp = 256: tile i holds heads [128 i, 128 i + 128) of the unit's position)
    const int boxes = 128 / p.boxh;
    for (int t = lane; t < 2 * boxes; t += 32) {
      const int half = t & 1;
      const int bx = t >> 1;
      const int row0 = 128 * i + bx * p.boxh;
      const int slot_abs = min(u.pb * p.pc + row0 / p.rp, u.count - 1);
      const int pos = min(max(load_pos(p, u.branch, u.b, slot_abs), 0), p.Sq - 1);
      const int row = (u.b * p.Sq + pos) * p.Hq + head0 + row0 % p.rp;
      tma_load_2d_hint(qdst + half * kHalfBytes + bx * p.boxh * 128, &p.q_map, bar, half * 64, row, pol);
    }
    return;
  }
  const int spt = 128 / p.rp;
  const int base = u.pb * p.pc + i * spt;  // absolute slot of the tile's first row
  auto pos_of = [&](int s) {
    return min(max(load_pos(p, u.branch, u.b, min(base + s, u.count - 1)), 0), p.Sq - 1);
  };
  for (int s = lane; s < spt; s += 32) {
    int lev = 0;
    for (int L = p.n_q3; L >= 1; --L) {
      const int b0 = s & ~((1 << L) - 1);
      const int b1 = b0 + (1 << L) - 1;
      // all slots of the block routed (no clamped repeats) and positions consecutive
      if (base + b1 < u.count && pos_of(b1) - pos_of(b0) == (1 << L) - 1) {
        lev = L;
        break;
      }
    }
    if ((s & ((1 << lev) - 1)) != 0) continue;  // not the first slot of its block
    const int pos = pos_of(s);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      if (lev == 0) {
        const int row = (u.b * p.Sq + pos) * p.Hq + head0;
        tma_load_2d_hint(qdst + half * kHalfBytes + s * p.rp * 128, &p.q_map, bar, half * 64, row, pol);
      } else {
        tma_load_3d_hint(qdst + half * kHalfBytes + s * p.rp * 128, &p.q_runs[lev - 1], bar, half * 64, head0,
                         u.b * p.Sq + pos, pol);
      }
    }
  }
}

// 2^x for a pair of arguments on the FMA pipe.  Cody-Waite style range
// reduction x = j + f with j = round(x) (the 1.5 * 2^23 shifter), f in
// [-0.5, 0.5]; 2^f by a degree-3 polynomial fitted for minimum maximal relative
// error on that interval (max relative error 7.5e-5, below the BF16 rounding that
// P receives); 2^j is added to the exponent field.  Arguments are clamped at
// -125 so the result stays a normal number: masked entries (-inf) give 2^-125
// instead of 0.  In a row with a legal key the entry that set the running max
// contributes 1 to the row sum, so these terms lie far below FP32 resolution; a
// row without any legal key is detected from its bounds in the epilogue and
// written as the reference writes it (O = 0/0 = NaN, LSE = log2(0) = -inf).
__device__ __forceinline__ void exp2_poly_pair(uint64_t x2, float& p0, float& p1) {
  float x0, x1;
  f2_unpack(x2, x0, x1);
  x0 = fmaxf(x0, -125.0f);
  x1 = fmaxf(x1, -125.0f);
  const uint64_t xc = f2_pack(x0, x1);
  const uint64_t shifter = f2_pack(12582912.0f, 12582912.0f);
  const uint64_t neg_shifter = f2_pack(-12582912.0f, -12582912.0f);
  const uint64_t minus_one = f2_pack(-1.0f, -1.0f);
  const uint64_t t = f2_add(xc, shifter);          // 1.5 * 2^23 + round(x)
  const uint64_t jf = f2_add(t, neg_shifter);      // round(x)
  const uint64_t f = f2_fma(jf, minus_one, xc);    // x - round(x)
  uint64_t p = f2_fma(f2_pack(0.05517097935080528f, 0.05517097935080528f), f,
                      f2_pack(0.24260970950126648f, 0.24260970950126648f));
  p = f2_fma(p, f, f2_pack(0.6932609677314758f, 0.6932609677314758f));
  p = f2_fma(p, f, f2_pack(0.9999281764030457f, 0.9999281764030457f));
  float t0, t1, q0, q1;
  f2_unpack(t, t0, t1);
  f2_unpack(p, q0, q1);
  // bits(t) = bits(shifter) + j and bits(shifter) * 2^23 vanishes mod 2^32
  p0 = __int_as_float(__float_as_int(t0) * (1 << 23) + __float_as_int(q0));
  p1 = __int_as_float(__float_as_int(t1) * (1 << 23) + __float_as_int(q1));
}

__device__ __forceinline__ float row_max64(const float* s) {
  float t[22];
#pragma unroll
  for (int i = 0; i < 21; ++i) t[i] = fmax3(s[3 * i], s[3 * i + 1], s[3 * i + 2]);
  t[21] = s[63];
  float u[8];
#pragma unroll
  for (int i = 0; i < 7; ++i) u[i] = fmax3(t[3 * i], t[3 * i + 1], t[3 * i + 2]);
  u[7] = t[21];
  return fmax3(fmax3(u[0], u[1], u[2]), fmax3(u[3], u[4], u[5]), fmaxf(u[6], u[7]));
}

// kRep: the launch also writes the replicated row-major outputs (p.n_rep > 0);
// kSplit: long full-causal units run as key-split pieces (p.pieces > 1) whose
// partial rows go to the scratch.  Separate instantiations, so the plain launch
// carries none of that code.
template <bool kRep, bool kSplit>
__global__ void __launch_bounds__(kThreads, 1) switch_prefill_kernel(const __grid_constant__ PrefillParams p) {
  if (p.gate != nullptr && *p.gate != 0) return;  // index validation failed: write nothing
#ifdef SWA_CYCLES
  const unsigned long long cycles_start = clock64();
#endif

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
  uint64_t* p_chunk = bars + SmemLayout::b_p_chunk;
  uint64_t* o_full = bars + SmemLayout::b_o_full;
  uint64_t* o_empty = bars + SmemLayout::b_o_empty;
  uint64_t* drain = bars + SmemLayout::b_drain;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSchedSlots; ++s) {
      mbar_init(&sched_full[s], 1);
      mbar_init(&sched_empty[s], 1 + 512);  // MMA lane 0 and the 512 softmax threads
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);  // committed after the unit's last S MMA of tile i
      mbar_init(&s_full[i], 1);
      mbar_init(&p_chunk[2 * i], 256);
      mbar_init(&p_chunk[2 * i + 1], 256);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 256);
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

  if (warp == 0) {
    // ------------------------------------------------------------------ scheduler + producer
    // Lane 0 takes work items from the global counter, every lane decodes the same
    // item, the unit is published through the ring for the MMA and softmax warps,
    // and the warp then issues the unit's TMA loads.
    int maxnpb0 = 0, maxnpb1 = 0;
    for (int b = 0; b < p.B; ++b) {
      maxnpb0 = max(maxnpb0, (min(branch_count(p, 0, b), p.idx_cap[0]) + p.pc - 1) / p.pc);
      maxnpb1 = max(maxnpb1, (min(branch_count(p, 1, b), p.idx_cap[1]) + p.pc - 1) / p.pc);
    }
    const int per_level = p.n_bg * p.nhb;
    const int total = (maxnpb0 * (kSplit ? p.pieces : 1) + maxnpb1) * per_level;
    auto fetch = [&](Unit& u) {
      u.valid = 0;
      while (true) {
        int it = 0;
        if (lane == 0) it = atomicAdd(p.counter, 1);
        it = __shfl_sync(0xffffffffu, it, 0);
        if (it >= total) break;
        if (decode_item<kSplit>(p, it, maxnpb0, maxnpb1, u)) break;
      }
    };
    uint32_t kv_it = 0;
    uint32_t q_use[2] = {0, 0};
    Tracer tr(lane == 0 ? 3 : -1);
    // The next unit is claimed from the counter only while this unit's last
    // kFetchAheadTiles + 1 key tiles are being loaded (several tiles before the MMA
    // warp reaches the unit's end, so the claim and its decode stay hidden).  A
    // claim at the start of the unit would hold the next item for the whole unit:
    // with few units per launch (a multi-GPU share) a long full-causal unit claimed
    // that way waited behind another long one and set the launch's length.
    Unit u;
    fetch(u);
    for (int k = 0;; ++k) {
      tr.ev(60, k);
      Unit un;
      un.valid = 0;
      bool fetched = !u.valid;  // nothing follows the end marker
      auto fetch_next = [&]() {
        if (!fetched) {
          fetch(un);
          fetched = true;
          tr.ev(61, k);
        }
      };
      const int slot = k % kSchedSlots;
      if (!mbar_wait(&sched_empty[slot], ((k / kSchedSlots) & 1) ^ 1, abort_flag)) break;
      if (lane == 0) {
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
        if (kSplit) dst->part = u.part;
        mbar_arrive(&sched_full[slot]);
      }
      __syncwarp();
      if (!u.valid) break;
      tr.ev(62, k);
      bool ok = true;
      if (u.n > 0) {
        auto load_kv = [&](int j, int kv) -> bool {
          const uint32_t s = kv_it % kStages;
          if (!mbar_wait(&kv_empty[s], ((kv_it / kStages) & 1) ^ 1, abort_flag)) return false;
          // one TMA box per tile (both 64-column halves), issued by lane 0 after it
          // arms the barrier.  (With the failure-detection test hook, CTA 0 never arms
          // or loads its second ring entry: the MMA warp's bounded wait on it runs out.)
          const bool withhold = p.test_withhold != 0 && blockIdx.x == 0 && kv_it == 1;
          if (lane == 0 && !withhold) {
            mbar_arrive_expect_tx(&kv_full[s], kTileBytes);
            uint8_t* dst = smem + SmemLayout::kv + s * kTileBytes;
            const CUtensorMap* map = kv == 0 ? &p.k_map : &p.v_map;
            tma_load_5d_hint(dst, map, &kv_full[s], 0, u.j0 * 64 + j * kBK, 0, u.g, u.b, l2_policy_evict_last());
          }
          __syncwarp();
          ++kv_it;
          return true;
        };
        auto load_q = [&](int i) -> bool {
          // Q_i is free once the previous unit's last S MMA of tile i has completed
          if (!mbar_wait(&q_empty[i], (q_use[i] & 1) ^ 1, abort_flag)) return false;
          tr.ev(63 + 2 * i, k);
          ++q_use[i];
          if (lane == 0) mbar_arrive_expect_tx(&q_full[i], kTileBytes);
          __syncwarp();
          q_tile_boxes(p, u, i, lane, smem + (i == 0 ? SmemLayout::q0 : SmemLayout::q1), &q_full[i]);
          tr.ev(64 + 2 * i, k);
          return true;
        };
        // ring order K_0, V_0, K_1, V_1, ...; the Q tiles go between K_0 and V_0 so
        // that K_0 streams in while the previous unit's epilogues still hold Q
        ok = load_kv(0, 0) && load_q(0) && load_q(1) && load_kv(0, 1);
        if (ok && u.n - 1 <= kFetchAheadTiles) fetch_next();
        for (int j = 1; j < u.n && ok; ++j) {
          ok = load_kv(j, 0) && load_kv(j, 1);
          if (ok && j >= u.n - 1 - kFetchAheadTiles) fetch_next();
        }
      }
      if (!ok) break;
      fetch_next();
      u = un;
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
    // The whole warp runs this loop (waits, descriptors); one elected lane issues
    // each tcgen05 instruction.
    constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, 128, false, true);
    const uint32_t q_addr[2] = {smem_u32(smem + SmemLayout::q0), smem_u32(smem + SmemLayout::q1)};
    const uint32_t kv_addr = smem_u32(smem + SmemLayout::kv);
    const uint32_t tm_s[2] = {tmem + 0, tmem + 128};
    const uint32_t tm_o[2] = {tmem + 256, tmem + 384};
    uint32_t kv_it = 0, q_use[2] = {0, 0}, p_use[2] = {0, 0}, o_use[2] = {0, 0};
    int k_sched = 0;
    bool ok = true;
    Tracer tr(lane == 0 ? 0 : -1);
    int step = 0;

    // Next unit with key tiles from the ring (units without any are consumed and skipped).
    auto next_unit = [&](Unit& u) -> bool {
      while (true) {
        const int slot = k_sched % kSchedSlots;
        if (!mbar_wait(&sched_full[slot], (k_sched / kSchedSlots) & 1, abort_flag)) { ok = false; return false; }
        read_unit<kSplit>(&units[slot], u);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sched_empty[slot]);
        ++k_sched;
        if (!u.valid) return false;
        if (u.n > 0) return true;
      }
    };
    // Descriptors are built once; a ring entry's descriptor is the base plus the
    // entry offset in the 14-bit start-address field (bytes >> 4).
    // The Q descriptors of all eight K = 16 steps of both tiles are fixed; a K ring
    // entry's eight are made when its load is waited for, off the path from a P
    // chunk to the next S MMA.
    uint64_t qd[2][8];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) qd[i][kk] = make_smem_desc_sw128(q_addr[i], 16, 1024) + k128_step_offset(kk);
    const uint64_t k_desc0 = make_smem_desc_sw128(kv_addr, 16, 1024);
    const uint64_t v_desc0 = make_smem_desc_sw128(kv_addr, kHalfBytes, 1024);
    uint64_t kd[8];
    auto k_descs = [&](uint32_t kstage) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) kd[kk] = k_desc0 + kstage * (kTileBytes >> 4) + k128_step_offset(kk);
    };
    auto issue_s = [&](int i) { umma_ss8_warp(tm_s[i], qd[i], kd, idesc_s); };
    // P V for one tile in two chunks: chunk c covers keys [64 c, 64 c + 64) (P columns
    // 32 c .. 32 c + 31, V rows in 2048-byte steps of 16 keys from 4 c), published by
    // the softmax before it exponentiates chunk c + 1.
    // S MMAs of one key step for tile i (K ring entry of the last k_descs call); after
    // the unit's last one, Q_i is released to the producer (the commit arrives once
    // these MMAs have read it).
    auto issue_s_step = [&](int i, bool last_of_unit) {
      issue_s(i);
      tc_commit_warp(&s_full[i]);
      if (last_of_unit) tc_commit_warp(&q_empty[i]);
    };
    // P V chunk c of tile i (waits for the chunk's P).
    auto issue_pv_chunk = [&](int i, int c, uint64_t vb, bool accumulate) -> bool {
      if (!mbar_wait(&p_chunk[2 * i + c], p_use[i] & 1, abort_flag)) { ok = false; return false; }
      tc_fence_after();
      umma_ts_k32_warp(tm_o[i], tm_s[i] + 32 * c, vb + (4 * c) * 128, idesc_o, (accumulate || c > 0) ? 1u : 0u);
      umma_ts_k32_warp(tm_o[i], tm_s[i] + 32 * c + 16, vb + (4 * c + 2) * 128, idesc_o, 1u);
      if (c == 1) ++p_use[i];
      return true;
    };

    Unit cur;
    bool have = next_unit(cur);
    if (have) {
      const uint32_t ks = kv_it % kStages;
      ok = ok && mbar_wait(&q_full[0], q_use[0] & 1, abort_flag);
      ok = ok && mbar_wait(&kv_full[ks], (kv_it / kStages) & 1, abort_flag);
      if (ok) {
        ++q_use[0];
        k_descs(ks);
        tc_fence_after();
        issue_s_step(0, cur.n == 1);
      }
      ok = ok && mbar_wait(&q_full[1], q_use[1] & 1, abort_flag);
      if (ok) {
        ++q_use[1];
        tc_fence_after();
        issue_s_step(1, cur.n == 1);
        tc_commit_warp(&kv_empty[ks]);
        ++kv_it;
      }
    }
    int j = 0;
    while (have && ok) {
      // invariant: S_0(j), S_1(j) of `cur` are issued.  Inside a unit the order is
      // PV_0(j), S_0(j+1), PV_1(j), S_1(j+1); at a unit's last step both P V MMAs go
      // first, then the next unit's S MMAs (S_i(0) overwrites the columns that hold
      // P_i of this step).  The waits for V_j and K_{j+1} (normally landed long ago)
      // come first, so that from the last P chunk of a tile to its next S MMA the
      // warp only issues MMAs.
      const bool last = j == cur.n - 1;
      const uint32_t vs = kv_it % kStages;
      tr.ev(1, step);
      if (!mbar_wait(&kv_full[vs], (kv_it / kStages) & 1, abort_flag)) { ok = false; break; }
      ++kv_it;
      uint32_t ks = 0;
      if (!last) {
        ks = kv_it % kStages;
        if (!mbar_wait(&kv_full[ks], (kv_it / kStages) & 1, abort_flag)) { ok = false; break; }
        ++kv_it;
        k_descs(ks);
      }
      tc_fence_after();
      tr.ev(2, step);
      if (j == 0) {
        if (!mbar_wait(&o_empty[0], (o_use[0] & 1) ^ 1, abort_flag)) { ok = false; break; }
        ++o_use[0];
      }
      const uint64_t vb = v_desc0 + vs * (kTileBytes >> 4);
      if (!issue_pv_chunk(0, 0, vb, j > 0)) break;
      tr.ev(3, step);
      if (!issue_pv_chunk(0, 1, vb, j > 0)) break;
      if (last) {
        tc_commit_warp(&o_full[0]);
      } else {
        issue_s_step(0, j + 1 == cur.n - 1);
      }
      tr.ev(4, step);
      if (j == 0) {
        if (!mbar_wait(&o_empty[1], (o_use[1] & 1) ^ 1, abort_flag)) { ok = false; break; }
        ++o_use[1];
      }
      if (!issue_pv_chunk(1, 0, vb, j > 0)) break;
      if (!issue_pv_chunk(1, 1, vb, j > 0)) break;
      tc_commit_warp(&kv_empty[vs]);
      if (!last) {
        issue_s_step(1, j + 1 == cur.n - 1);
        tc_commit_warp(&kv_empty[ks]);
        tr.ev(5, step);
        ++j;
      } else {
        tc_commit_warp(&o_full[1]);
        have = next_unit(cur);
        if (!ok || !have) break;
        tr.ev(7, step);
        j = 0;
        const uint32_t k0s = kv_it % kStages;
        if (!mbar_wait(&q_full[0], q_use[0] & 1, abort_flag)) { ok = false; break; }
        tr.ev(8, step);
        ++q_use[0];
        if (!mbar_wait(&kv_full[k0s], (kv_it / kStages) & 1, abort_flag)) { ok = false; break; }
        tr.ev(9, step);
        ++kv_it;
        k_descs(k0s);
        tc_fence_after();
        issue_s_step(0, cur.n == 1);
        tr.ev(17, step);
        if (!mbar_wait(&q_full[1], q_use[1] & 1, abort_flag)) { ok = false; break; }
        tr.ev(18, step);
        ++q_use[1];
        tc_fence_after();
        issue_s_step(1, cur.n == 1);
        tc_commit_warp(&kv_empty[k0s]);
      }
      tr.ev(6, step);
      ++step;
    }
    // drain: wait until every MMA issued by this warp has completed
    tc_commit_warp(drain);
    volatile int dummy = 0;
    mbar_wait(drain, 0, &dummy);
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    // Warps 2-17: tile = (warp - 2) / 8.  A warp may only access its TMEM lane
    // quarter warp % 4; the two warps of a tile with the same quarter take its lanes
    // 0..15 and 16..31 (block hb).  Within a warp, thread l (< 16) and thread l + 16
    // share row t = 32 q + 16 hb + l (16-lane TMEM loads): thread half 0 holds keys
    // [0, 32) and [64, 96) of every key tile, half 1 keys [32, 64) and [96, 128).
    // The row max of a key step and the row sum of a unit are exchanged between the
    // two threads of a row with one warp shuffle: no shared memory, no barrier.
    const int grp = (warp - 2) >> 2;             // 0..3
    const int tile = grp >> 1;
    const int hb = grp & 1;
    const int half = lane >> 4;
    const int lane_base = (warp & 3) * 32 + 16 * hb;
    const int t = lane_base + (lane & 15);       // row within the tile = TMEM lane
    const uint32_t tm_s = tmem + 128 * tile + (static_cast<uint32_t>(lane_base) << 16);
    const uint32_t tm_o = tmem + 256 + 128 * tile + (static_cast<uint32_t>(lane_base) << 16);
    const int R = 128 * tile + t;                  // row within the unit
    const int slot_in_unit = R / p.rp;
    const int head_in_group_off = R % p.rp;
    const int r = p.Hq / p.Hkv;
    const float sl2 = p.scale_log2;
    const float m_init = -1073741824.0f * sl2;     // reference initial row max (-2^30), scaled
    const uint64_t sl2x2 = f2_pack(sl2, sl2);
    uint32_t s_use = 0, o_use = 0;
    bool ok = true;
    Tracer tr(t == 0 && half == 0 ? 1 + tile : -1);
    for (int k = 0; ok; ++k) {
      const int slot = k % kSchedSlots;
      if (!mbar_wait(&sched_full[slot], (k / kSchedSlots) & 1, abort_flag)) break;
      Unit u;
      read_unit<kSplit>(&units[slot], u);
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
          const uint4 nan4 = make_uint4(nan_pair, nan_pair, nan_pair, nan_pair);
          for (int t = -1; t < (kRep ? p.n_rep : 0); ++t) {
            __nv_bfloat16* ob = t < 0 ? p.out : p.rep_out[t];
            float* lb = t < 0 ? p.lse : p.rep_lse[t];
            if (ob == nullptr) continue;
            const int64_t row = t < 0 ? orow : replica_row(p, u.b, qpos, head);
            uint4* dst0 = reinterpret_cast<uint4*>(ob + row * 128 + 32 * half);
            uint4* dst1 = reinterpret_cast<uint4*>(ob + row * 128 + 64 + 32 * half);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              dst0[c] = nan4;
              dst1[c] = nan4;
            }
            if (half == 0) lb[row] = -INFINITY;
          }
        }
        continue;
      }
      float m = m_init;
      float l = 0.0f;   // partial row sum over this thread's keys
      for (int j = 0; j < u.n; ++j) {
        tr.ev(10, s_use + 1);
        if (!mbar_wait(&s_full[tile], s_use & 1, abort_flag)) { ok = false; break; }
        tr.ev(11, s_use + 1);
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld_16x2_x32(tm_s, sr + 0);        // keys 32 half + [0, 32)
        tmem_ld_16x2_x32(tm_s + 64, sr + 32);  // keys 64 + 32 half + [0, 32)
        tmem_ld_wait();
        reg_fence32(sr + 0);
        reg_fence32(sr + 32);
        float* s = reinterpret_cast<float*>(sr);
        const int k0 = u.j0 * 64 + j * kBK;
        const bool need_mask = !(rb.lo <= k0 && k0 + kBK <= rb.hi);
        // legal keys among the 32 keys from `base`: one 32-bit mask, then one
        // predicated select per entry
        auto key_mask = [&](int base) -> uint32_t {
          const int a = min(max(rb.lo - base, 0), 32);
          const int b = max(min(rb.hi - base, 32), a);
          const uint32_t hi_bits = b >= 32 ? ~0u : ((1u << b) - 1u);
          const uint32_t lo_bits = a >= 32 ? ~0u : ((1u << a) - 1u);
          return hi_bits & ~lo_bits;
        };
        const int kb0 = k0 + 32 * half, kb1 = k0 + 64 + 32 * half;
        if (need_mask) {
          const uint32_t v0 = key_mask(kb0), v1 = key_mask(kb1);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            s[e] = select_or_neg_inf(v0, 1u << e, s[e]);
            s[32 + e] = select_or_neg_inf(v1, 1u << e, s[32 + e]);
          }
        }
        tr.ev(12, s_use + 1);
        // partial max, exchanged with the thread of the same row (lane ^ 16)
        const float pmax = row_max64(s);
        const float m_tile = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, 16)) * sl2;
        tr.ev(15, s_use + 1);
        ++s_use;
        bool rescale = false;
        float alpha = 1.0f;
        if (m == m_init) {
          m = fmaxf(m, m_tile);
        } else if (m_tile > m + kRescaleThreshold) {
          alpha = ex2_approx(m - m_tile);
          l *= alpha;
          m = m_tile;
          rescale = true;
        }
        if (__any_sync(0xffffffffu, rescale)) {
          // this thread's columns of the O row (P V of earlier key tiles, all
          // complete) *= alpha, before any P of this key step is published
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t orr[16];
            const uint32_t ta = tm_o + (c >> 1) * 64 + (c & 1) * 32;  // columns [32 c', +32) of the two halves
            tmem_ld_16x2_x16(ta, orr);
            tmem_ld_wait();
            reg_fence16(orr);
#pragma unroll
            for (int e = 0; e < 16; ++e) orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
            tmem_st_16x2_x16(ta, orr);
          }
        }
        const uint64_t negm2 = f2_pack(-m, -m);
        uint64_t acc[4] = {0, 0, 0, 0};
        // chunk c = keys [64 c, 64 c + 64) of the tile (this thread: 32 of them),
        // P pairs into columns 32 c + 16 half .. + 15, published as soon as it is in
        // TMEM so the P V MMAs of chunk 0 run while chunk 1 is exponentiated.
        // Chunk 1's scores are read from TMEM again (columns 64..127, which chunk
        // 0's P does not reach), so their registers are free meanwhile.
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
          uint32_t sr1[32];
          const float* sc = s;
          if (c == 1) {
            tmem_ld_16x2_x32(tm_s + 64, sr1);
            tmem_ld_wait();
            reg_fence32(sr1);
            float* s1 = reinterpret_cast<float*>(sr1);
            if (need_mask) {
              const uint32_t v1 = key_mask(kb1);
#pragma unroll
              for (int e = 0; e < 32; ++e) s1[e] = select_or_neg_inf(v1, 1u << e, s1[e]);
            }
            sc = s1 - 32;
          }
#pragma unroll
          for (int qq = 0; qq < 16; ++qq) {
            const int q = 16 * c + qq;
            const uint64_t x2 = f2_fma(f2_pack(sc[2 * q], sc[2 * q + 1]), sl2x2, negm2);
            float p0, p1;
            if ((q & 3) == 3) {
              exp2_poly_pair(x2, p0, p1);
            } else {
              float x0, x1;
              f2_unpack(x2, x0, x1);
              p0 = ex2_approx(x0);
              p1 = ex2_approx(x1);
            }
            acc[q & 3] = f2_add(acc[q & 3], f2_pack(p0, p1));
            pk[qq] = pack_bf16x2(p0, p1);
          }
          tmem_st_16x2_x16(tm_s + 32 * c, pk);
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(&p_chunk[2 * tile + c]);
        }
        tr.ev(16, s_use);
        tr.ev(13, s_use);
        float a0, a1, b0, b1, c0, c1, d0, d1;
        f2_unpack(acc[0], a0, a1);
        f2_unpack(acc[1], b0, b1);
        f2_unpack(acc[2], c0, c1);
        f2_unpack(acc[3], d0, d1);
        l += ((a0 + a1) + (b0 + b1)) + ((c0 + c1) + (d0 + d1));
      }
      if (!ok) break;
      // epilogue: O / l -> BF16 written straight from registers with coalesced
      // stores: each thread packs its 64 columns (eight 16-byte chunks: columns
      // 32 half + 8 j for j < 4, 64 + 32 half + 8 (j - 4) for j >= 4), the eight lanes
      // of a lane group transpose their 8 x 8 chunks with three xor butterflies (lane
      // L then holds chunk L % 8 of the group's eight rows), so one store instruction
      // writes two 64-byte pieces of four rows.  LSE in log2 units.
      tr.ev(20, s_use);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      if (!mbar_wait(&o_full[tile], o_use & 1, abort_flag)) { ok = false; break; }
      ++o_use;
      tr.ev(21, s_use);
      if constexpr (kSplit) {
        if (u.part >= 0) {
          // a key-split piece: the row's partial O / l (FP32) and partial LSE over the
          // piece's keys [klo, khi) into the scratch; a row without a legal key in
          // the piece gets O = 0 and LSE = -inf (weight 0 in the merge)
          const int klo = u.j0 * 64, khi = klo + u.n * kBK;
          const bool none = max(rb.lo, klo) >= min(rb.hi, khi);
          const float sc = none ? 0.0f : 1.0f / l;
          float* po = p.part_o + (static_cast<int64_t>(u.part) * 256 + R) * 128 + 32 * half;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t orr[32];
            tmem_ld_16x2_x32(tm_o + 64 * c, orr);
            tmem_ld_wait();
            reg_fence32(orr);
            if (valid_row) {
#pragma unroll
              for (int e = 0; e < 8; ++e)
                reinterpret_cast<float4*>(po + 64 * c)[e] =
                    make_float4(__uint_as_float(orr[4 * e]) * sc, __uint_as_float(orr[4 * e + 1]) * sc,
                                __uint_as_float(orr[4 * e + 2]) * sc, __uint_as_float(orr[4 * e + 3]) * sc);
            }
          }
          tc_fence_before();
          mbar_arrive(&o_empty[tile]);
          if (half == 0 && valid_row)
            p.part_lse[static_cast<int64_t>(u.part) * 256 + R] = none ? -INFINITY : lg2_approx(l) + m;
          continue;
        }
      }
      // A row whose key range is empty (metadata start >= end, or a local row at
      // t >= Skv + W - 1) has row sum 0 in the reference (swiattn_gqa_prefill.py:201-206,
      // swiattn_gqa_prefill_varlen.py:236-241): O = 0/0 and LSE = log2(0) + m.
      const bool no_keys = rb.hi <= rb.lo;
      const float inv_l = no_keys ? __int_as_float(0x7FC00000) : 1.0f / l;
      const int64_t rrow = (kRep && valid_row) ? replica_row(p, u.b, qpos, head) : -1;
      if (half == 0 && valid_row) {
        const float lse_v = no_keys ? -INFINITY : lg2_approx(l) + m;
        if (!kRep || p.lse != nullptr) p.lse[orow] = lse_v;
        if constexpr (kRep) {
          for (int t = 0; t < p.n_rep; ++t) p.rep_lse[t][rrow] = lse_v;
        }
      }
      tc_fence_after();
      uint32_t ch[8][4];  // ch[j]: chunk j of this thread's columns as BF16 pairs
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t orr[32];
        tmem_ld_16x2_x32(tm_o + 64 * c, orr);
        tmem_ld_wait();
        reg_fence32(orr);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          ch[4 * c + e / 4][e % 4] = pack_bf16x2(__uint_as_float(orr[2 * e]) * inv_l,
                                                 __uint_as_float(orr[2 * e + 1]) * inv_l);
      }
      tc_fence_before();
      mbar_arrive(&o_empty[tile]);  // O_i fully read: the next unit's P V may overwrite it
#pragma unroll
      for (int bit = 2; bit >= 0; --bit) {
        const int msk = 1 << bit;
        const bool upper = (lane & msk) != 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j & msk) continue;
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint32_t x = upper ? ch[j][w] : ch[j | msk][w];
            const uint32_t y = __shfl_xor_sync(0xffffffffu, x, msk);
            if (upper) {
              ch[j][w] = y;
            } else {
              ch[j | msk][w] = y;
            }
          }
        }
      }
      const int64_t my_row = (valid_row && (!kRep || p.out != nullptr)) ? orow : -1;
      const int my_chunk = lane & 7;
      const int col = my_chunk < 4 ? 32 * half + 8 * my_chunk : 64 + 32 * half + 8 * (my_chunk - 4);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int src = (lane & ~7) + j;  // lane holding row j of this group
        const int64_t grow = __shfl_sync(0xffffffffu, my_row, src);
        if (grow >= 0) {
          const uint4 val = make_uint4(ch[j][0], ch[j][1], ch[j][2], ch[j][3]);
          st_global_v4_hint(p.out + grow * 128 + col, val, l2_policy_evict_first());
        }
      }
      if constexpr (kRep) {
        // the same chunks into every row-major replica (this GPU's or a peer's
        // memory, written over NVLink), at the row's global position
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int src = (lane & ~7) + j;
          const int64_t grow = __shfl_sync(0xffffffffu, rrow, src);
          if (grow >= 0) {
            const uint4 val = make_uint4(ch[j][0], ch[j][1], ch[j][2], ch[j][3]);
            for (int t = 0; t < p.n_rep; ++t) *reinterpret_cast<uint4*>(p.rep_out[t] + grow * 128 + col) = val;
          }
        }
      }
      tr.ev(22, s_use);
    }
    // replicas in peer memory: make this thread's stores visible system-wide before
    // the kernel completes (the caller's barrier then publishes them to the peers)
    if constexpr (kRep) __threadfence_system();
  }

  // ------------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(p.status, kStatusTimeout);
#ifdef SWA_CYCLES
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_swa_cycles[blockIdx.x] = clock64() - cycles_start;
#endif
}

// Combines the key-split pieces of one unit per block (grid: split_pb_cap x nhb x
// units; blocks of units that are not split return at once): for every routed row
// of the unit, LSE = log2(sum_s 2^LSE_s) and O = sum_s 2^(LSE_s - LSE) O_s over its
// pieces s, written as BF16 at the row's position; a row without a legal key in
// any piece gets O = NaN, LSE = -inf (the reference's 0/0 and log2(0)).  A warp
// per row, four columns per lane.
__global__ void __launch_bounds__(256) merge_pieces_kernel(const __grid_constant__ PrefillParams p) {
  if (p.gate != nullptr && *p.gate != 0) return;
  const int rr = blockIdx.x, hb = blockIdx.y, bgi = blockIdx.z;  // rr: rank from the last position block
  const int bg = p.bg_list != nullptr ? p.bg_list[bgi] : bgi;
  const int b = bg / p.Hkv;
  const int g = bg % p.Hkv;
  const int cnt = min(branch_count(p, 0, b), p.idx_cap[0]);
  const int pb = (cnt + p.pc - 1) / p.pc - 1 - rr;
  if (pb < 0) return;
  const int first_slot = pb * p.pc;
  int j0, n, np, len, used;
  unit_tiles(p, 0, b, first_slot, cnt, j0, n);
  split_pieces(p, n, np, len, used);
  if (np <= 1) return;
  const int64_t base = ((static_cast<int64_t>(bgi) * p.nhb + hb) * p.split_pb_cap + rr) * p.pieces;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = p.Hq / p.Hkv;
  for (int R = warp; R < 256; R += 8) {
    const int slot_abs = first_slot + R / p.rp;
    if (slot_abs >= cnt) continue;
    const int qpos = load_pos(p, 0, b, slot_abs);
    if (qpos < 0 || qpos >= p.Sq) continue;
    const int head = g * r + hb * p.rp + R % p.rp;
    const int64_t orow = (static_cast<int64_t>(b) * p.Sq + qpos) * p.Hq + head;
    float M = -INFINITY;
    for (int s = 0; s < used; ++s) M = fmaxf(M, p.part_lse[(base + s) * 256 + R]);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float lse = -INFINITY;
    if (M == -INFINITY) {
      acc = make_float4(NAN, NAN, NAN, NAN);
    } else {
      float sum = 0.0f;
      for (int s = 0; s < used; ++s) sum += exp2f(p.part_lse[(base + s) * 256 + R] - M);
      lse = M + log2f(sum);
      for (int s = 0; s < used; ++s) {
        const float w = exp2f(p.part_lse[(base + s) * 256 + R] - lse);
        if (w == 0.0f) continue;
        const float4 o = reinterpret_cast<const float4*>(p.part_o + ((base + s) * 256 + R) * 128)[lane];
        acc.x += w * o.x;
        acc.y += w * o.y;
        acc.z += w * o.z;
        acc.w += w * o.w;
      }
    }
    const __nv_bfloat162 lo2 = __floats2bfloat162_rn(acc.x, acc.y);
    const __nv_bfloat162 hi2 = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 packed;
    packed.x = *reinterpret_cast<const uint32_t*>(&lo2);
    packed.y = *reinterpret_cast<const uint32_t*>(&hi2);
    reinterpret_cast<uint2*>(p.out + orow * 128)[lane] = packed;
    if (lane == 0) p.lse[orow] = lse;
  }
}

template <bool kRep, bool kSplit>
cudaError_t launch_instance(const PrefillParams& params, int num_sms, cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(switch_prefill_kernel<kRep, kSplit>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  switch_prefill_kernel<kRep, kSplit><<<num_sms, kThreads, kSmemBytes, stream>>>(params);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill(const PrefillParams& params, int num_sms, cudaStream_t stream) {
  if (params.n_rep > 0) return launch_instance<true, false>(params, num_sms, stream);
  if (params.pieces > 1) return launch_instance<false, true>(params, num_sms, stream);
  return launch_instance<false, false>(params, num_sms, stream);
}

cudaError_t launch_merge_pieces(const PrefillParams& params, cudaStream_t stream) {
  if (params.pieces <= 1) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(params.split_pb_cap), static_cast<unsigned>(params.nhb),
                  static_cast<unsigned>(params.n_bg));
  merge_pieces_kernel<<<grid, 256, 0, stream>>>(params);
  return cudaGetLastError();
}

SplitPlan plan_split(int n_units, int nhb, int pc, int full_cap, int local_cap, int Skv, int window, int num_sms,
                     int request_tiles) {
  SplitPlan s{0, 1, 0, 0};
  const int64_t n_max = (static_cast<int64_t>(Skv) + kBK - 1) / kBK;  // most key tiles a unit can have
  const int64_t pb_cap = (static_cast<int64_t>(full_cap) + pc - 1) / pc;
  const int64_t uf = pb_cap * n_units * nhb;                                        // full-branch units
  const int64_t ul = ((static_cast<int64_t>(local_cap) + pc - 1) / pc) * n_units * nhb;  // local-branch units
  if (uf == 0 || n_max < 2) return s;
  int64_t tiles = request_tiles;
  if (tiles <= 0) {
    // Split only when the longest full-causal unit would outlast the average work
    // per SM by half: full units taken as n_max / 2 tiles on average, local units
    // as the window plus a unit's position span.
    const int64_t t_local = std::min<int64_t>(n_max, (static_cast<int64_t>(window) + pc + 2 * kBK - 2) / kBK);
    const double est = (0.5 * static_cast<double>(uf) * static_cast<double>(n_max) +
                        static_cast<double>(ul) * static_cast<double>(t_local)) /
                       static_cast<double>(num_sms > 0 ? num_sms : 1);
    if (n_max < 64 || static_cast<double>(n_max) <= 1.5 * est) return s;
    tiles = std::max<int64_t>(32, static_cast<int64_t>(std::ceil(est)));
  }
  if (n_max <= tiles) return s;
  const int64_t pieces = (n_max + tiles - 1) / tiles;
  // scratch slots for the k_cap longest full-branch units of each (unit, head
  // block): as many as the lists can hold, within kSplitScratchBudget bytes
  constexpr int64_t kSplitScratchBudget = int64_t(512) << 20;
  const int64_t per_rank = static_cast<int64_t>(nhb) * n_units * pieces * kSplitSlotBytes;
  const int64_t k_cap = std::min<int64_t>(pb_cap, kSplitScratchBudget / per_rank);
  if (k_cap < 1 || pieces > (int64_t(1) << 20)) return s;
  const int64_t slots = k_cap * nhb * n_units * pieces;
  s.tiles = static_cast<int>(tiles);
  s.pieces = static_cast<int>(pieces);
  s.pb_cap = static_cast<int>(k_cap);
  s.bytes = static_cast<size_t>(slots * kSplitSlotBytes);
  return s;
}

uint32_t prefill_smem_bytes() { return kSmemBytes; }

#ifdef SWA_TRACE
// Points the cycle tracer of CTA 0 at a device buffer of 5 x 2 x 8192 uint64
// (one region per recorder) or, with nullptr, turns it off.
extern "C" int swa_dev_trace_set(void* buf) {
  unsigned long long* ptr = static_cast<unsigned long long*>(buf);
  return static_cast<int>(cudaMemcpyToSymbol(g_swa_trace, &ptr, sizeof(ptr)));
}
#endif

#ifdef SWA_CYCLES
// Copies the per-CTA cycle counts of the last launch (n <= 1024) to host memory.
extern "C" int swa_dev_cycles(unsigned long long* host, int n) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, g_swa_cycles, sizeof(unsigned long long) * n));
}
#endif

}  // namespace swa
