// Internal declarations shared by the CUDA translation units of libswattn_b200.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace swa {

// Bits of the device status word (int32).  The index-validation kernels set the
// first group; the prefill kernel sets kStatusTimeout when a bounded wait gave up.
enum : int32_t {
  kStatusFullRange = 1 << 0,   // full list: index outside [0, seq_len)
  kStatusFullOrder = 1 << 1,   // full list: not strictly increasing
  kStatusLocalRange = 1 << 2,  // local list: index outside [0, seq_len)
  kStatusLocalOrder = 1 << 3,  // local list: not strictly increasing
  kStatusFullPad = 1 << 4,     // full list ([B, N] form): -1 padding not trailing
  kStatusLocalPad = 1 << 5,    // local list ([B, N] form): -1 padding not trailing
  kStatusCover = 1 << 6,       // per-batch counts do not add up to the sequence length
  kStatusTimeout = 1 << 16,    // a device-side wait exceeded its limit
};

constexpr int kMaxQRunMaps = 7;
constexpr int kMaxReplicas = 8;  // row-major output copies one prefill launch can write

struct __align__(64) PrefillParams {
  CUtensorMap q_map;  // 2-D {128, B*Sq*Hq}, box {64, boxh}, 128B swizzle
  // 3-D {128, Hq, B*Sq} views of q with box {64, rp, 2^(L+1)}: 2^(L+1) consecutive
  // positions x rp heads in one TMA box (L < n_q3; n_q3 = log2(128 / rp), rp <= 64)
  CUtensorMap q_runs[kMaxQRunMaps];
  int n_q3;
  CUtensorMap k_map;  // 5-D {64, Skv, 2, Hkv, B} (column half as a dimension), box {64, 128, 2, 1, 1}, 128B swizzle
  CUtensorMap v_map;
  const int32_t* idx[2];       // routed positions per branch: [B, idx_stride]
  int idx_stride[2];
  int idx_cap[2];              // valid slots per row are < min(count, idx_cap)
  const int32_t* counts;       // device counts (nullable): counts[branch * cs_branch + b * cs_batch]
  int cs_branch, cs_batch;
  int count_scalar[2];         // counts for B == 1 when `counts` is null
  const int32_t* starts[2];    // metadata: full_starts, local_starts (nullable)
  const int32_t* ends;         // metadata: causal_ends (nullable: fixed-length masks)
  const int32_t* bg_list;      // (b * Hkv + g) units handled by this launch (nullable: all)
  int n_bg;
  __nv_bfloat16* out;          // [B, Sq, Hq, 128]
  float* lse;                  // [B, Sq, Hq]
  int* counter;                // work counter, zero at launch
  int* status;                 // status word (kStatus* bits)
  const int* gate;             // nullable; non-zero => the launch does nothing
  int B, Sq, Skv, Hq, Hkv, window;
  float scale_log2;
  int rp;    // query heads per position in a unit (power of two dividing Hq/Hkv)
  int pc;    // positions per unit = 256 / rp
  int nhb;   // head blocks per KV group = (Hq/Hkv) / rp
  int boxh;  // rows per Q TMA box = min(rp, 128)
  int test_withhold;  // failure-detection test hook: CTA 0 withholds its second K/V tile load
  // Replicated row-major outputs (multi-GPU driver; launches with Hkv == 1 over
  // unit-major inputs): batch b of the launch is global unit unit_gid[b] =
  // b_g * rep_hkv + g_g, and every output row is also stored to rep_out[t] /
  // rep_lse[t] (t < n_rep; [Bg, Sq, rep_hkv * Hq, 128] / [Bg, Sq, rep_hkv * Hq]),
  // this GPU's memory or a peer's.  `out` / `lse` may then be null (not written).
  int n_rep;
  int rep_hkv;
  const int32_t* unit_gid;
  __nv_bfloat16* rep_out[kMaxReplicas];
  float* rep_lse[kMaxReplicas];
  // Key-split pieces of long full-causal units (pieces == 1: off).  A full-branch
  // unit of n > split_tiles key tiles runs as np = ceil(n / split_tiles) pieces of
  // ceil(n / np) tiles, each a work item of its own (on whichever CTA takes it);
  // a piece writes every routed row's partial O / l (FP32) and partial LSE into
  // the scratch slot ((bgi * nhb + hb) * split_pb_cap + rr) * pieces + piece, rr =
  // the unit's rank from the last position block of its branch (only units with
  // rr < split_pb_cap are split), and merge_pieces_kernel combines the pieces.
  int pieces;        // work items per full-branch unit: ceil(max tiles / split_tiles)
  int split_tiles;
  int split_pb_cap;  // longest units per (unit, head block) with scratch slots
  float* part_o;     // [slots, 256, 128]
  float* part_lse;   // [slots, 256]
};

// Scratch bytes of one key-split slot: partial LSE and partial O of 256 rows.
constexpr int64_t kSplitSlotBytes = 256 * 4 + 256 * 128 * 4;

// Plan of a key-split prefill launch (swa_prefill_split_plan): tiles == 0 means
// no split.
struct SplitPlan {
  int tiles;
  int pieces;
  int pb_cap;
  size_t bytes;  // scratch: partial LSE of every slot, then partial O (256-byte aligned)
};
SplitPlan plan_split(int n_units, int nhb, int pc, int full_cap, int local_cap, int Skv, int window, int num_sms,
                     int request_tiles);

cudaError_t launch_prefill(const PrefillParams& params, int num_ctas, cudaStream_t stream);
// Combines the pieces of every split unit of a launch (after launch_prefill on
// the same stream).
cudaError_t launch_merge_pieces(const PrefillParams& params, cudaStream_t stream);

// Decode step: one query token per sequence against its KV cache.
struct __align__(64) DecodeParams {
  // BF16 cache: 4-D {128, Hkv, Smax, B}, box {64, 1, 64, 1}, 128B swizzle.
  // FP8 cache (fp8 != 0): bytes, 4-D {128, Hkv, Smax, B}, box {128, 1, 64, 1}.
  CUtensorMap k_map;
  CUtensorMap v_map;
  int fp8;                  // K/V cache in FP8 e4m3 with per-(b, KV head) scales
  const float* k_scale;     // [B, Hkv] (fp8 only): K = k_cache * k_scale
  const float* v_scale;     // [B, Hkv] (fp8 only): V = v_cache * v_scale
  const __nv_bfloat16* q;   // [B, Hq, 128]
  const int32_t* seq_lens;  // [B] cached keys including the new token
  const uint8_t* route;     // [B] non-zero = full attention
  __nv_bfloat16* out;       // [B, Hq, 128]
  float* lse;               // [B, Hq]
  float* part_o;            // [B, Hkv, nhb, splits, 16, 128] split partials
  float* part_ml;           // [B, Hkv, nhb, splits, 16, 2] (max, sum) of each partial row
  int32_t* status;
  int B, Smax, Hq, Hkv, r, nhb, splits, split_keys, window;
  float scale_log2;
};
cudaError_t launch_decode(const DecodeParams& params, cudaStream_t stream);

// Prefill backward: dQ, dK, dV of both branches.
//
// Packed rows: the routed rows of (branch, b, g) in packed order (row R = slot
// R / r of the branch's list, query head g r + R % r), R < idx_stride[branch] * r,
// branch 0's regions first: packed index = (branch ? pk_n0 : 0)
// + (b * Hkv + g) * idx_stride[branch] * r + R.  The pack pass writes, per packed
// row, Q and dO (BF16, 128 dims; zeros for absent rows), the record {lo, hi,
// LSE bits, D bits} (legal key range, empty when the row is absent or has no
// legal key; D = rowsum(dO * O)) and the position (-1 when absent).
struct __align__(64) BwdParams {
  CUtensorMap k_map;         // 4-D {128, Hkv, Skv, B}, box {64, 1, 64, 1}, 128B swizzle
  CUtensorMap v_map;
  CUtensorMap qp_map;        // 2-D {128, packed rows}, box {64, 64}, 128B swizzle
  CUtensorMap dop_map;
  CUtensorMap rec_map;       // 2-D int32 {4, packed rows}, box {4, 64}, no swizzle
  const __nv_bfloat16 *q, *k, *v, *o, *dout;
  const float* lse;          // [B, Sq, Hq] forward LSE (log2 units)
  const int32_t* idx[2];     // [B, stride] routed positions of each branch, -1 padded
  int idx_stride[2];
  const int32_t* counts;     // [B, 2] (n_full, n_local)
  const int32_t* starts[2];  // metadata (nullable)
  const int32_t* ends;
  __nv_bfloat16 *dq, *dk, *dv;
  // workspace: packed rows
  int4* rec;
  int32_t* rpos;
  __nv_bfloat16 *qp, *dop;
  int64_t pk_n0;             // packed rows of branch 0
  int64_t pk_rows;           // packed rows of both branches
  int B, Sq, Skv, Hq, Hkv, r, window;
  float scale_log2, scale;   // softmax scale in log2 units and in natural units
  int nblk[2];               // dQ pass: 128-row blocks of each branch per (batch, KV group)
  int32_t* status;           // kStatusTimeout when a bounded wait gave up
};
// Workspace bytes of the backward: status word, then the packed rows (records,
// positions, Q, dO), each section 256-byte aligned.
size_t backward_workspace_bytes(int B, int Hq, int full_stride, int local_stride);
// Points the packed-row fields and the status word of `p` (B, Hq, idx_stride
// set) into a workspace of backward_workspace_bytes().
void bind_backward_workspace(BwdParams& p, void* workspace);
cudaError_t launch_backward(const BwdParams& params, int num_sms, cudaStream_t stream);
uint32_t decode_smem_bytes();

// Record the message returned by swa_last_error_string() on this thread.
void set_last_error(const char* msg);
uint32_t prefill_smem_bytes();

// Workspace (int32 elements) the compaction takes to split rows over several
// CTAs; 0 when every row fits one CTA.  With ws == nullptr the compaction runs
// one CTA per row.
int64_t compact_workspace_elems(int B, int S);
cudaError_t launch_compact_mask(const uint8_t* mask, int B, int S, int32_t* full, int32_t* local,
                                int32_t* counts, int32_t* ws, cudaStream_t stream);

// Router output element types of swa_compact_router (values of SWA_ROUTER_*).
constexpr int kRouterBf16 = 1;
constexpr int kRouterF32 = 2;
cudaError_t launch_compact_router(const void* router, int dtype, int pair, float threshold, int B, int S,
                                  int32_t* full, int32_t* local, int32_t* counts, int32_t* ws, cudaStream_t stream);

cudaError_t launch_prepare_indices(const int32_t* idx, int B, int N, int seq_len, int padded_rows, int cap,
                                   int32_t* padded, int32_t* count, int32_t* status, int range_bit, int order_bit,
                                   int pad_bit, cudaStream_t stream);

cudaError_t launch_check_cover(const int32_t* counts, int B, int seq_len, int32_t* status, cudaStream_t stream);

cudaError_t launch_build_metadata(const int32_t* cu_seqlens, int nseg, int q_len, int kv_len, int window,
                                  int32_t* q_positions, int32_t* kv_positions, int32_t* q_segment_ids,
                                  int32_t* kv_segment_ids, int32_t* full_starts, int32_t* local_starts,
                                  int32_t* causal_ends, cudaStream_t stream);

}  // namespace swa
