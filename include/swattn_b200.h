/*
 * libswattn_b200 -- C ABI of the B200 (sm_100a) Switch Attention GQA prefill path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, a cudaStream_t; NULL = legacy default stream), enqueues its
 * work on that stream and returns 0 on success or a negative SWA_E* code.  No
 * entry point allocates memory or synchronises the stream.  On error,
 * swa_last_error_string() describes the failure (thread-local).
 *
 * Layouts (all row-major, contiguous):
 *   q    bf16 [B, Sq, Hq, 128]        k, v  bf16 [B, Skv, Hkv, 128]
 *   out  bf16 [B, Sq, Hq, 128]        lse   fp32 [B, Sq, Hq]  (log2 domain)
 *   index lists int32 [B, stride]: routed positions, strictly increasing.
 *
 * Reference interfaces replaced (YushengZhao/SwitchAttentionKernels):
 *   swa_compact_mask      <- build_switch_query_indices   swiattn_gqa_prefill_varlen.py:306-322
 *   swa_compact_router    <- the router step before it (outside the reference,
 *                            README.md:85) fused with the compaction
 *   swa_compact_*_ws      <- the same two, rows split over several CTAs
 *   swa_prepare_indices   <- _prepare_indices             swiattn_gqa_prefill_varlen.py:271-304
 *   swa_check_cover       <- coverage check               swiattn_gqa_prefill_varlen.py:390-393
 *   swa_build_metadata    <- build_switch_attention_metadata (imported at
 *                            swiattn_gqa_prefill_varlen.py:27, used at :353-359)
 *   swa_prefill_forward   <- both _switch_gqa_prefill_branch launches of
 *                            switch_gqa_prefill_forward     swiattn_gqa_prefill_varlen.py:395-446
 *                            (kernels swiattn_gqa_prefill.py:8-214,
 *                             swiattn_gqa_prefill_varlen.py:33-249)
 */
#ifndef SWATTN_B200_H_
#define SWATTN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SWA_OK 0
#define SWA_E_INVALID (-1)     /* bad argument (shape, pointer, alignment)      */
#define SWA_E_CUDA (-2)        /* a CUDA runtime call failed                    */
#define SWA_E_UNSUPPORTED (-3) /* e.g. head_dim != 128, not an sm_100 device    */
#define SWA_E_TMA (-4)         /* tensor-map encoding failed                    */

/* Status-word bits written by the validation kernels and the prefill kernel. */
#define SWA_STATUS_FULL_RANGE (1 << 0)
#define SWA_STATUS_FULL_ORDER (1 << 1)
#define SWA_STATUS_LOCAL_RANGE (1 << 2)
#define SWA_STATUS_LOCAL_ORDER (1 << 3)
#define SWA_STATUS_FULL_PAD (1 << 4)
#define SWA_STATUS_LOCAL_PAD (1 << 5)
#define SWA_STATUS_COVER (1 << 6)
#define SWA_STATUS_TIMEOUT (1 << 16)

/* ABI version of this header (1). */
int swa_abi_version(void);

/* Description of the last error on the calling thread ("" if none). */
const char* swa_last_error_string(void);

/* Number of SMs of `device` (the persistent grid size), or a negative code. */
int swa_num_sms(int device);

/* Failure-detection test hook; no counterpart in the reference.  While `on` is
 * non-zero, every swa_prefill_forward launch makes its first CTA withhold one
 * K/V tile load, so the MMA issuer's bounded wait for that tile runs out: the
 * launch returns with SWA_STATUS_TIMEOUT in workspace[1] after about one second,
 * having released its tensor memory, and the CUDA context stays usable.  Not for
 * production use; off by default. */
void swa_test_withhold_kv_load(int on);

/* Compact a routing mask (uint8/bool [B, S], non-zero = full attention) into
 * the increasing full / local position lists full[B, S], local[B, S]; entries
 * past each row's count are -1.  counts[2*b] = n_full, counts[2*b+1] = n_local.
 * Replaces build_switch_query_indices (swiattn_gqa_prefill_varlen.py:306-322),
 * which handles B = 1 only. */
int swa_compact_mask(const uint8_t* mask, int B, int S, int32_t* full, int32_t* local, int32_t* counts,
                     void* stream);

/* Router output -> routing decision -> compaction in one kernel (no mask
 * buffer).  The reference leaves the router outside the kernel and compacts a
 * bool mask (README.md:85, build_switch_query_indices
 * swiattn_gqa_prefill_varlen.py:306-322); this entry point takes the router's
 * output instead.  router: dtype SWA_ROUTER_BF16 or SWA_ROUTER_F32, contiguous
 *   pair = 0: [B, S]    one score per token, full iff score > threshold;
 *   pair = 1: [B, S, 2] logits (local, full), full iff
 *             logit_full - logit_local > threshold (0 = argmax, ties local).
 * Values are compared in FP32; NaN routes to local.  Outputs as
 * swa_compact_mask. */
#define SWA_ROUTER_BF16 1
#define SWA_ROUTER_F32 2
int swa_compact_router(const void* router, int dtype, int pair, float threshold, int B, int S, int32_t* full,
                       int32_t* local, int32_t* counts, void* stream);

/* The compactions above with a caller-provided int32 workspace of at least
 * swa_compact_workspace_elems(B, S) elements (0 when every row fits one CTA):
 * rows longer than one 4096-token chunk are then split over several CTAs in
 * two launches (per-chunk counts, then scan and write), instead of one CTA per
 * row.  Results are identical.  SWA_E_INVALID when the workspace is too small. */
int64_t swa_compact_workspace_elems(int B, int S);
int swa_compact_mask_ws(const uint8_t* mask, int B, int S, int32_t* full, int32_t* local, int32_t* counts,
                        int32_t* workspace, int64_t workspace_elems, void* stream);
int swa_compact_router_ws(const void* router, int dtype, int pair, float threshold, int B, int S, int32_t* full,
                          int32_t* local, int32_t* counts, int32_t* workspace, int64_t workspace_elems,
                          void* stream);

/* Prefill backward (no counterpart in the reference, which is forward only,
 * swiattn_gqa_prefill_varlen.py:14): dq [B, Sq, Hq, 128], dk, dv [B, Skv, Hkv, 128]
 * (bf16) of the forward's output, from o, its lse (fp32 [B, Sq, Hq], log2
 * units) and dout (bf16, like o).  Index lists: -1 padded [B, stride] rows with
 * counts[2*b] = n_full, counts[2*b+1] = n_local (as swa_compact_mask writes
 * them); metadata as in swa_prefill_forward (nullable).  workspace: 16-byte
 * aligned, at least swa_backward_workspace_bytes(B, Hq, full_stride,
 * local_stride) bytes (the routed rows' Q and dO in packed order with their key
 * ranges, LSE and rowsum(dout * o): about 532 bytes per routed (position, head)
 * slot of the lists); its first int32 receives SWA_STATUS_TIMEOUT if a bounded
 * device wait gave up. */
size_t swa_backward_workspace_bytes(int B, int Hq, int full_stride, int local_stride);
int swa_prefill_backward(const void* q, const void* k, const void* v, const void* o, const float* lse,
                         const void* dout, const int32_t* full_idx, const int32_t* local_idx, int full_stride,
                         int local_stride, const int32_t* counts, const int32_t* full_starts,
                         const int32_t* local_starts, const int32_t* causal_ends, void* dq, void* dk, void* dv,
                         int B, int Sq, int Skv, int Hq, int Hkv, int head_dim, int window, float scale_log2,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Decode step (no counterpart in the reference, which is prefill only): one
 * new query token per sequence against its KV cache, routed per sequence.
 *   q [B, Hq, 128] bf16; k_cache, v_cache [B, Smax, Hkv, 128] bf16;
 *   seq_lens int32 [B]: cached keys of sequence b including the new token
 *   (1 <= L <= Smax; the new token's K/V sit at row L - 1);
 *   route uint8 [B]: non-zero = full causal attention (keys [0, L)), zero =
 *   sliding window (keys [max(0, L - window), L));
 *   out [B, Hq, 128] bf16, lse [B, Hq] fp32 (log2 domain, as the prefill).
 * workspace: at least swa_decode_workspace_bytes(B, Smax, Hq, Hkv) bytes,
 * 16-byte aligned; int32 workspace[0] receives the status bits
 * (SWA_STATUS_TIMEOUT) of the launch. */
size_t swa_decode_workspace_bytes(int B, int Smax, int Hq, int Hkv);
int swa_decode_forward(const void* q, const void* k_cache, const void* v_cache, const int32_t* seq_lens,
                       const uint8_t* route, void* out, float* lse, int B, int Smax, int Hq, int Hkv,
                       int head_dim, int window, float scale_log2, void* workspace, size_t workspace_bytes,
                       void* stream);

/* The decode step over an FP8 KV cache (no counterpart in the reference): as
 * swa_decode_forward with k_cache / v_cache [B, Smax, Hkv, 128] in FP8 e4m3 (one
 * byte per element) and per-(sequence, KV head) FP32 scales k_scale, v_scale
 * [B, Hkv]: the attention uses K = k_cache * k_scale and V = v_cache * v_scale.
 * Half the cache bytes of the BF16 step, which is HBM-bound.  The products run
 * in FP16 (the e4m3 values convert exactly; q is converted from BF16 and must
 * lie within the FP16 range; P is rounded to FP16).  Same workspace as
 * swa_decode_workspace_bytes(B, Smax, Hq, Hkv). */
int swa_decode_forward_fp8(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                           const float* v_scale, const int32_t* seq_lens, const uint8_t* route, void* out, float* lse,
                           int B, int Smax, int Hq, int Hkv, int head_dim, int window, float scale_log2,
                           void* workspace, size_t workspace_bytes, void* stream);

/* Capacity-bucket preparation and validation of one index list per batch row
 * (replaces _prepare_indices, swiattn_gqa_prefill_varlen.py:271-304).
 *   idx [B, N]; trailing_pad = 0: all N entries are routed rows (the reference
 *   form, count = N); trailing_pad = 1: -1 entries are trailing padding.
 *   padded [B, cap] (nullable) receives the list with -1 fill; count [B].
 *   Violations OR range_bit / order_bit / pad_bit into *status. */
int swa_prepare_indices(const int32_t* idx, int B, int N, int seq_len, int trailing_pad, int cap,
                        int32_t* padded, int32_t* count, int32_t* status, int range_bit, int order_bit,
                        int pad_bit, void* stream);

/* counts [2, B] (full row then local row): ORs SWA_STATUS_COVER into *status
 * when count_full[b] + count_local[b] != seq_len for some b
 * (swiattn_gqa_prefill_varlen.py:390-393). */
int swa_check_cover(const int32_t* counts, int B, int seq_len, int32_t* status, void* stream);

/* Per-row key bounds for packed varlen prefill.  cu_seqlens int32 [nseg + 1]
 * (nullable: one sequence).  Writes the seven SwitchAttentionMetadata vectors
 * of lengths (q_len, kv_len, q_len, kv_len, q_len, q_len, q_len). */
int swa_build_metadata(const int32_t* cu_seqlens, int nseg, int q_len, int kv_len, int window,
                       int32_t* q_positions, int32_t* kv_positions, int32_t* q_segment_ids,
                       int32_t* kv_segment_ids, int32_t* full_starts, int32_t* local_starts,
                       int32_t* causal_ends, void* stream);

/* Both Switch Attention branches of causal GQA prefill in one persistent launch.
 *   full_idx / local_idx : int32 [B, *_stride]; row b holds the first counts
 *                          of routed positions (B == 1 with counts == NULL:
 *                          count_full / count_local are used).
 *   full_cap / local_cap : number of readable slots per row (<= stride).
 *   counts               : int32 device counts (nullable when B == 1): [2, B]
 *                          (full row, then local row) or, with
 *                          counts_batch_major = 1, [B, 2] as written by
 *                          swa_compact_mask.
 *   full_starts, local_starts, causal_ends : int32 [Sq] varlen bounds
 *                          (all NULL: fixed-length masks key <= t and
 *                          t - window + 1 <= key <= t).
 *   bg_list / n_bg       : (b * Hkv + g) work units to compute (NULL: all B*Hkv),
 *                          used by the multi-GPU driver to shard units.
 *   gate                 : nullable device int32; non-zero makes the launch a no-op
 *                          (set by the validation kernels).
 *   workspace            : >= 16 bytes of device memory; workspace[0] is the work
 *                          counter (zeroed by this call on `stream`),
 *                          workspace[1] receives SWA_STATUS_TIMEOUT on a device-side
 *                          wait timeout.  Launches that overlap on the GPU need
 *                          distinct workspaces.
 * Requires head_dim == 128, Hq % Hkv == 0, window > 0, 16-byte aligned q/k/v. */
int swa_prefill_forward(const void* q, const void* k, const void* v, const int32_t* full_idx,
                        const int32_t* local_idx, int full_stride, int local_stride, int full_cap, int local_cap,
                        const int32_t* counts, int counts_batch_major, int count_full, int count_local,
                        const int32_t* full_starts,
                        const int32_t* local_starts, const int32_t* causal_ends, const int32_t* bg_list, int n_bg,
                        void* out, float* lse, int B, int Sq, int Skv, int Hq, int Hkv, int head_dim, int window,
                        float scale_log2, const int32_t* gate, int32_t* workspace, size_t workspace_bytes,
                        void* stream);

/* Key-split plan for swa_prefill_forward_split (no counterpart in the reference,
 * whose full-causal branch gives each 64-row query tile one CTA over its whole
 * key prefix, swiattn_gqa_prefill.py:95-105).  A full-branch work unit whose key
 * range spans more than *split_tiles 128-key tiles is then run as several pieces
 * of about equal length on different SMs, and a merge kernel combines their
 * partial O and LSE.  This lets a launch with few, long full-causal units (a
 * multi-GPU shard of one or two (batch, KV group) units of a 131K-token
 * sequence) end with the average work per SM instead of its longest unit.
 * request_tiles > 0 asks for pieces of about that many tiles; 0 lets the plan
 * decide from the launch shape (split only when the longest possible
 * full-causal unit would outlast the estimated work per SM by half; scratch kept
 * under 1 GiB).  n_bg: units of the launch (0: all B * Hkv).  num_sms: SMs of
 * the device.  Returns the scratch bytes the launch needs and writes the piece
 * length to *split_tiles (0 and 0: no split).  Needs no GPU. */
size_t swa_prefill_split_plan(int B, int Skv, int Hq, int Hkv, int full_cap, int local_cap, int n_bg, int window,
                              int num_sms, int request_tiles, int* split_tiles);

/* swa_prefill_forward with long full-causal units split over several CTAs
 * (see swa_prefill_split_plan; split_tiles == 0 is swa_prefill_forward).
 * scratch: 16-byte aligned device memory, normally the plan's bytes: it holds
 * slots for the longest full-causal units of every (unit, head block), as many
 * as fit (at least one each, or the call fails); longer-ranked units run whole.
 * Every routed row of a split unit gets its partial O (FP32) and LSE there from
 * each piece, then a second kernel on `stream` writes O and LSE.  Results match the
 * unsplit launch to rounding (each piece rounds P to BF16 against its own
 * running max).  Not combinable with replicated outputs.  Launches that overlap
 * on the GPU need distinct workspaces and scratch buffers. */
int swa_prefill_forward_split(const void* q, const void* k, const void* v, const int32_t* full_idx,
                              const int32_t* local_idx, int full_stride, int local_stride, int full_cap, int local_cap,
                              const int32_t* counts, int counts_batch_major, int count_full, int count_local,
                              const int32_t* full_starts, const int32_t* local_starts, const int32_t* causal_ends,
                              const int32_t* bg_list, int n_bg, void* out, float* lse, int B, int Sq, int Skv, int Hq,
                              int Hkv, int head_dim, int window, float scale_log2, const int32_t* gate,
                              int32_t* workspace, size_t workspace_bytes, int split_tiles, void* scratch,
                              size_t scratch_bytes, void* stream);

/* Prefill over a rank's unit-major inputs with its output replicated in
 * row-major form (multi-GPU driver; no counterpart in the reference, which has
 * no distributed code -- its per-(batch, head) grid, swiattn_gqa_prefill.py:69,
 * admits the (batch, KV group) split).  The launch is swa_prefill_forward with
 * Hkv = 1 over B units: q [B, Sq, Hq, 128], k/v [B, Skv, 1, 128], -1 padded
 * [B, *_stride] index lists with counts [B, 2] (batch-major, as swa_compact_mask
 * writes them), metadata as there.  Unit b of the launch is global unit
 * unit_gid[b] (device int32 [B]) = b_g * rep_hkv + g_g of a [Bg, Sq, rep_hkv * Hq,
 * 128] problem, and every output row is stored into each of the n_rep (1..8)
 * row-major buffers rep_out[t] (bf16 [Bg, Sq, rep_hkv * Hq, 128]) and
 * rep_lse[t] (fp32 [Bg, Sq, rep_hkv * Hq]) at its global position: this GPU's
 * memory or a peer's (peer pointers from symmetric / IPC-mapped memory, written
 * over NVLink by the kernel's epilogue).  out / lse (the unit-major result) may
 * be NULL.  Rows of other units in the replicas are left untouched; making the
 * peers' writes visible (a barrier after the launch on every rank) is the
 * caller's.  Workspace and status as swa_prefill_forward. */
int swa_prefill_forward_replicated(const void* q, const void* k, const void* v, const int32_t* full_idx,
                                   const int32_t* local_idx, int full_stride, int local_stride,
                                   const int32_t* counts, const int32_t* full_starts, const int32_t* local_starts,
                                   const int32_t* causal_ends, const int32_t* unit_gid, int B, int Sq, int Skv, int Hq,
                                   int head_dim, int window, float scale_log2, int rep_hkv, int n_rep,
                                   void* const* rep_out, float* const* rep_lse, void* out, float* lse,
                                   int32_t* workspace, size_t workspace_bytes, void* stream);

/* Unit-major <-> row-major moves of the multi-GPU driver (no counterpart in the
 * reference, which has no distributed code; its per-(batch, head) grid,
 * swiattn_gqa_prefill.py:69, admits the (batch, KV group) split these serve).
 * A unit is u = b * hkv + g.  Unit-major: [n_slots, S, chunk_bytes]; slot i
 * holds unit unit_of_slot[i] (device int32; -1 = padding slot, skipped).
 * Row-major: [B, S, row_bytes] with unit (b, g) at byte offset g * chunk_bytes of
 * each row (e.g. O: chunk_bytes = r * 128 * 2, row_bytes = Hq * 128 * 2; LSE:
 * r * 4 and Hq * 4).  swa_scatter_units: unit-major src -> row-major dst (the
 * permute after an all-gather of every rank's units); swa_gather_units: row-major
 * src -> unit-major dst (a rank's unit slices).  chunk_bytes, row_bytes and the
 * pointers must be multiples of 4; 16 gives 16-byte vector moves.  At most 65535
 * slots. */
/* Context-parallel K/V exchange (no counterpart in the reference; the reference's
 * metadata path addresses a gathered key axis, swiattn_gqa_prefill_varlen.py:179-182):
 * copy `bytes` bytes from src (this GPU) to each of the n_dst (<= 8) destinations
 * dsts[i] (this GPU's or a peer's memory, e.g. every rank's symmetric-memory K/V
 * buffer at the chunk's token offset), each 16-byte word loaded once and stored to
 * every destination with plain stores.  bytes, src and every dsts[i] must be
 * multiples of 16.  Ordering against the peers is the caller's (a device barrier
 * of all ranks before and after). */
int swa_broadcast_bytes(const void* src, size_t bytes, void* const* dsts, int n_dst, void* stream);

int swa_scatter_units(const void* src, const int32_t* unit_of_slot, int n_slots, int S, int hkv, int chunk_bytes,
                      int row_bytes, void* dst, void* stream);
int swa_gather_units(const void* src, const int32_t* unit_of_slot, int n_slots, int S, int hkv, int chunk_bytes,
                     int row_bytes, void* dst, void* stream);

/* Allocation-free batched prefill.  No counterpart in the reference: it exists
 * for callers that must not allocate device memory when they run attention --
 * e.g. a plugin whose host framework owns all device memory and passes only
 * input and output buffers, or a serving loop held to a fixed memory budget in
 * which cudaMalloc (and the device synchronisation it can cause) is not allowed.
 * Same computation as swa_prefill_forward on -1 padded [B, *_stride] index
 * lists, including index validation, with all scratch (work counter, status
 * words, per-row counts) kept in a 16 KB array inside the library on each GPU
 * that loads it (held until the process exits).  Limits and behaviour:
 *   - 1 <= B <= swa_noalloc_max_batch() (2046); larger batches get SWA_E_INVALID;
 *   - nothing is allocated; the scratch is cleared on `stream` by every call;
 *   - every call on a device shares that one array, so calls that can overlap on
 *     the GPU (different streams, or a second call before the first finished on
 *     another stream) race -- serialise them on one stream;
 *   - the first call on a device resolves the array's device address (with that
 *     device current); make that first call before any stream capture (a lookup
 *     that fails returns SWA_E_CUDA and is retried by the next call);
 *   - status_out (nullable, device int32[2]) receives the validation bits
 *     (SWA_STATUS_FULL_* / LOCAL_* / COVER; a non-zero value means nothing was
 *     computed) and the kernel status bits (SWA_STATUS_TIMEOUT). */
int swa_noalloc_max_batch(void);
int swa_prefill_forward_noalloc(const void* q, const void* k, const void* v, const int32_t* full_idx,
                                const int32_t* local_idx, int full_stride, int local_stride,
                                const int32_t* full_starts, const int32_t* local_starts, const int32_t* causal_ends,
                                void* out, float* lse, int B, int Sq, int Skv, int Hq, int Hkv, int head_dim,
                                int window, float scale_log2, int32_t* status_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SWATTN_B200_H_ */
