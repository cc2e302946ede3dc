/*
 * mxfa_b200.h -- C ABI of libmxfa_b200.so, the sm_100a (B200) kernels behind
 * MXFlashAttn's decode and prefill hot path.
 *
 * Conventions
 *  - Every entry point is stream-ordered and asynchronous on `stream` (a
 *    cudaStream_t passed as void*; NULL = legacy default stream).  None of
 *    them synchronises the device or reads device memory on the host, so a
 *    caller may record them inside a CUDA graph.
 *  - The caller owns and allocates every buffer, including split workspaces
 *    (sizes from the *_workspace_bytes helpers).  Pointers are raw device
 *    pointers to contiguous row-major tensors.
 *  - Return value: MXFA_OK (0) on success; MXFA_ERR_UNSUPPORTED (-1) for a
 *    configuration the kernels do not cover (the same -1 the reference's
 *    launchers return); MXFA_ERR_INVALID (-2) for a bad argument;
 *    MXFA_ERR_CUDA (-3) when the launch itself failed.  mxfa_last_error()
 *    returns a thread-local description of the last non-zero status.
 *  - Element type: `bf16` = 1 for bfloat16, 0 for float16.  Arithmetic is
 *    fp32 (softmax, accumulation); outputs are rounded to nearest-even.
 *  - Stateless and re-entrant; the only module state is the device-side
 *    error word read by mxfa_read_error_flags().
 */
#ifndef MXFA_B200_H_
#define MXFA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MXFA_OK 0
#define MXFA_ERR_UNSUPPORTED (-1)
#define MXFA_ERR_INVALID (-2)
#define MXFA_ERR_CUDA (-3)

/* Device error flags (bitwise OR) raised by kernels instead of faulting. */
#define MXFA_FLAG_PAGE_OUT_OF_RANGE 0x1u  /* block-table entry outside [0, num_pages) */
#define MXFA_FLAG_TABLE_TOO_NARROW 0x2u   /* sequence longer than block_table width * page size */
#define MXFA_FLAG_WAIT_TIMEOUT 0x4u       /* a bounded pipeline wait gave up */
#define MXFA_FLAG_DENSE_OVERFLOW 0x8u     /* dense-cache append past the cache capacity */
#define MXFA_FLAG_BAD_ORDER 0x10u         /* a length order entry outside [0, B) (that row ran its own index) */

/* Library identity.  No reference counterpart (the reference's pybind
 * modules expose no version); used by the ctypes loader. */
int mxfa_abi_version(void);

/* Thread-local text of the last failing call (empty string if none).
 * Replaces the TORCH_CHECK messages of csrc_native/m1_binding.cpp:74,113. */
const char* mxfa_last_error(void);

/* 1 when the current CUDA device is sm_100 and the kernels can launch,
 * else 0.  Replaces `is_available()` of the ATen extension
 * (csrc/mxmac/attention_forward.cpp:98-100), which always returned true. */
int mxfa_is_available(void);

/* Read (and clear) the device error flags of the current device.
 * Synchronises the device: diagnostics and tests only, never in a hot path. */
int mxfa_read_error_flags(unsigned int* flags);

/* ------------------------------------------------------------------ decode */

/* Reference-compatible split-KV paged decode: same arguments, layouts and
 * return codes as the MetaX launcher it replaces,
 * mxfa_paged_decode_split_launch (csrc_native/m1_kernel.cpp:1206-1222).
 *   q   [B, 1, HQ, D]          k, v  [P, PS, HKV, D]      (bf16 or fp16)
 *   bt  int32 [B, BTW]         sl    int32 [B]
 *   out [B, 1, HQ, D]          ows   f32 [B, HQ, NP, D]   mdws f32 [B, HQ, NP, 2]
 * Chunk z covers positions [z*c_len, (z+1)*c_len) of each sequence; the
 * partials hold the unnormalised sum of p*v, the log2-domain running max m
 * and d = sum 2^(s - m), exactly the state the reference's split_combine
 * (m1_kernel.cpp:862-888) merges, and this call runs that combine too.
 * Guards as the reference: D in {64,128}, HQ % HKV == 0, GQ in {2,4,8},
 * NP >= 1, else -1.  `um` (the reference's softmax-variant switch, 0/1/2)
 * is ignored, as the reference launcher never rejects it either: every
 * variant is served by the same overflow-safe online softmax here.
 * Page indices are NOT bounded on this entry: the reference ABI carries no
 * page count, so the tensor maps span every slot row a 32-bit index can
 * name, and a corrupt block-table entry reads outside the caches (as it
 * would in the reference).  Callers that cannot vouch for their tables use
 * mxfa_kvcache_attention_launch, whose num_pages bounds every entry
 * (out-of-range entries read zeros and raise MXFA_FLAG_PAGE_OUT_OF_RANGE). */
int mxfa_paged_decode_split_launch(const void* q, const void* k, const void* v, const void* bt,
                                   const void* sl, void* out, void* ows, void* mdws, float scale,
                                   int B, int HQ, int HKV, int D, int PS, int BTW, int bf16, int NP,
                                   int c_len, int um, void* stream);

/* Bytes of split workspace (partials + (m,d) pairs) for `rows` query rows
 * (rows = B * Sq * HQ) and NP splits.  No reference counterpart: the
 * reference binding allocated these buffers itself (m1_binding.cpp:94-97). */
size_t mxfa_split_workspace_bytes(int rows, int D, int NP);

/* Split plan for flash_attn_with_kvcache on this GPU: number of splits and
 * chunk length (positions) for sequences of at most `max_len` tokens, sized
 * to the device's SM count.  Replaces the NP / c_len heuristic of the vLLM
 * hook (integrations/vllm/vllm_plugin.py:271-276). */
int mxfa_kvcache_plan(int B, int Sq, int HQ, int HKV, int D, int max_len, int* num_splits,
                      int* chunk_len);

/* KV-cache attention, the device path of flash_attn_with_kvcache
 * (mxflashattn/api.py:151-286; reference semantics mxflashattn/reference.py:88-139
 * with the append done separately by mxfa_kv_append_launch).
 *   q        [B, Sq, HQ, D]
 *   k_cache  paged [P, PS, HKV, D] (block_table != NULL) or dense [B, PS, HKV, D]
 *   seqlens  int32 [B]: cached lengths BEFORE this call's append; the call
 *            attends to seqlens[b] + append_len tokens
 *   out      [B, Sq, HQ, D];  lse optional f32 [B, Sq, HQ] (natural log)
 *   workspace f32, >= mxfa_split_workspace_bytes(B*Sq*HQ, D, num_splits)
 *            bytes when num_splits > 1 (may be NULL when num_splits == 1)
 * causal is bottom-right aligned (query i sees keys <= L - Sq + i).  Any
 * GQ = HQ / HKV is accepted; D in {64, 128}. */
int mxfa_kvcache_attention_launch(const void* q, const void* k_cache, const void* v_cache,
                                  const int32_t* block_table, const int32_t* seqlens, void* out,
                                  float* lse, void* workspace, size_t workspace_bytes, int B, int Sq,
                                  int HQ, int HKV, int D, int PS, int BTW, int num_pages,
                                  int append_len, int num_splits, int chunk_len, int causal,
                                  int bf16, float scale, void* stream);

/* Counter array for the single-launch split path: one unsigned per
 * (sequence, KV head, query-row group), i.e. B * HKV * ceil(Sq*GQ / g) * 4
 * bytes with g = 8 for Sq*GQ <= 8, else 16.  The caller zeroes it once after
 * allocating; every launch leaves it zero again. */
size_t mxfa_split_counter_bytes(int B, int Sq, int HQ, int HKV);

/* mxfa_kvcache_attention_launch in ONE kernel launch when the plan splits:
 * each split CTA publishes its partial state, counts itself on its unit's
 * counter, and the last one merges the unit's partials into out / lse (the
 * combine of m1_kernel.cpp:862-888 run inside the decode launch, removing
 * the second launch of m1_kernel.cpp:1000).  `counters` (see
 * mxfa_split_counter_bytes) must be zero on entry and is zero again when the
 * launch completes; launches that share a counter array must be ordered (one
 * stream, or events).  Unsplit plans ignore it. */
int mxfa_kvcache_attention_counted_launch(const void* q, const void* k_cache, const void* v_cache,
                                          const int32_t* block_table, const int32_t* seqlens, void* out,
                                          float* lse, void* workspace, size_t workspace_bytes,
                                          unsigned int* counters, int B, int Sq, int HQ, int HKV, int D, int PS,
                                          int BTW, int num_pages, int append_len, int num_splits,
                                          int chunk_len, int causal, int bf16, float scale, void* stream);

/* mxfa_kvcache_attention_counted_launch over e4m3 caches (FP8 KV, half the
 * decode bytes).  k_cache / v_cache hold float8_e4m3fn [.., PS, HKV, 128]
 * (head dim 128 only); the attended values are k_cache * k_scale and
 * v_cache * v_scale, both positive and finite.  q and out are bf16 (bf16=1)
 * or fp16.  Tiles are widened to f16 exactly and both products run in f16 on
 * the tensor cores, so q must stay within the f16 range.  `counters` may be
 * NULL (separate combine launch when the plan splits).  No reference
 * counterpart: FP8 KV was planned in docs/V1.5_OPTIMIZATION_PLAN.md:583-670
 * of the reference and never built there. */
int mxfa_kvcache_attention_fp8_launch(const void* q, const void* k_cache, const void* v_cache,
                                      const int32_t* block_table, const int32_t* seqlens, void* out,
                                      float* lse, void* workspace, size_t workspace_bytes,
                                      unsigned int* counters, int B, int Sq, int HQ, int HKV, int D, int PS,
                                      int BTW, int num_pages, int append_len, int num_splits, int chunk_len,
                                      int causal, int bf16, float scale, float k_scale, float v_scale,
                                      void* stream);

/* Plan once per step, run per layer.  The decode kernel runs a batch's
 * sequences longest first (1 < B <= 512): without an order every CTA ranks
 * all B lengths before its first block-table read, on every layer.
 * mxfa_kvcache_length_order_launch writes that order once (order[rank] =
 * sequence, int32 [B], longest first, ties by index) from seqlens on the
 * device; mxfa_kvcache_attention_ordered_launch then takes it in place of the
 * ranking.  The order only schedules: lengths are always read from seqlens,
 * so an order computed for other lengths of the same batch costs speed, not
 * correctness; an entry outside [0, B) raises MXFA_FLAG_BAD_ORDER and that
 * grid row runs its own index.  The ordered launch is
 * mxfa_kvcache_attention_counted_launch (counters may be NULL: separate
 * combine when the plan splits) or, with kv_fp8 = 1,
 * mxfa_kvcache_attention_fp8_launch, plus length_order (NULL: the kernel
 * ranks).  No reference counterpart (the reference launches the sequences in
 * index order, m1_kernel.cpp:970-1021). */
int mxfa_kvcache_length_order_launch(const int32_t* seqlens, int B, int32_t* order, void* stream);
int mxfa_kvcache_attention_ordered_launch(const void* q, const void* k_cache, const void* v_cache,
                                          const int32_t* block_table, const int32_t* seqlens,
                                          const int32_t* length_order, void* out, float* lse, void* workspace,
                                          size_t workspace_bytes, unsigned int* counters, int B, int Sq, int HQ,
                                          int HKV, int D, int PS, int BTW, int num_pages, int append_len,
                                          int num_splits, int chunk_len, int causal, int bf16, float scale,
                                          int kv_fp8, float k_scale, float v_scale, void* stream);

/* mxfa_kvcache_attention_launch with the append fused into the same launch:
 * the append of reference.py:108-122 (what mxfa_kv_append_launch does) plus
 * the attention over the grown cache, in one kernel.  k_new, v_new
 * [B, append_len, HKV, D] are written into k_cache / v_cache by the CTA that
 * reads those positions, then attended to.  seqlens still holds the lengths
 * before the append and is not modified (advance it with
 * mxfa_seqlens_add_launch).  Up to 16 query rows per KV head (Sq * GQ <= 16,
 * every single-token decode); larger shapes return MXFA_ERR_UNSUPPORTED and
 * need the separate append.  `counters` as in
 * mxfa_kvcache_attention_counted_launch, or NULL for a separate combine
 * launch.  No reference counterpart as one entry point: the reference
 * appended on the host (reference.py:117-122). */
int mxfa_kvcache_append_attention_launch(const void* q, void* k_cache, void* v_cache,
                                         const int32_t* block_table, const int32_t* seqlens, void* out,
                                         float* lse, void* workspace, size_t workspace_bytes,
                                         unsigned int* counters, const void* k_new, const void* v_new, int B,
                                         int Sq, int HQ, int HKV, int D, int PS, int BTW, int num_pages,
                                         int append_len, int num_splits, int chunk_len, int causal, int bf16,
                                         float scale, void* stream);

/* ---- Context-parallel decode with the exchange fused over peer memory ----
 * No reference counterpart (the reference runs on one device).  A group of
 * `world` ranks (one process per GPU) each hold a contiguous range of every
 * sequence's pages.  Per call:
 *   mxfa_cp_decode_launch  split decode of the local range; the merging CTA of
 *                          each (sequence, KV head) writes its normalised
 *                          (O, LSE) records into EVERY rank's exchange buffer
 *                          (plain NVLink stores), each 32-bit value paired
 *                          with the step's tag in one 64-bit word;
 *   mxfa_cp_merge_launch   on each rank: wait (bounded) until all ranks'
 *                          words carry the step's tag, LSE-merge the records
 *                          in rank order, write out / lse.
 * This replaces the NCCL all-gather of the records.  Exchange buffers come
 * from mxfa_peer_alloc (zeroed cudaMalloc) and are mapped on the other ranks
 * with mxfa_peer_export / mxfa_peer_import (CUDA IPC; no multicast).  One
 * buffer serves every layer: a device-side epoch advances per call and
 * alternates two halves of the buffer.  All ranks must issue the same
 * sequence of calls.  A rank that stops participating makes the others'
 * merge time out after 1 s (MXFA_FLAG_WAIT_TIMEOUT). */
size_t mxfa_cp_buffer_bytes(int world, int B, int HQ, int HKV, int D);
int mxfa_peer_alloc(size_t bytes, void** ptr);
int mxfa_peer_free(void* ptr);
int mxfa_peer_export(void* ptr, void* handle /* 64 bytes */);
int mxfa_peer_import(const void* handle /* 64 bytes */, void** ptr);
int mxfa_peer_close(void* ptr);
/* peer_bufs: device array of `world` exchange-buffer addresses as seen from
 * this rank (entry `rank` is the local buffer).  counters: as in
 * mxfa_kvcache_attention_counted_launch.  One query token per sequence. */
int mxfa_cp_decode_launch(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                          const int32_t* seqlens, void* out, float* lse, void* workspace, size_t workspace_bytes,
                          unsigned int* counters, const unsigned long long* peer_bufs, int rank, int world, int B,
                          int HQ, int HKV, int D, int PS, int BTW, int num_pages, int num_splits, int chunk_len,
                          int bf16, float scale, void* stream);
int mxfa_cp_merge_launch(void* local_buf, void* out, float* lse, int world, int B, int HQ, int HKV, int D, int bf16,
                         void* stream);
/* Both steps from one call: the decode kernel's merging CTA of each unit also
 * waits (bounded) for every rank's records of that unit and merges its rows into
 * out / lse, so a layer is one launch.  That CTA holds its SM while it waits,
 * so this is done only when the grid's units (B x HKV) are fewer than the
 * CTAs the GPU holds at once; otherwise the call launches the decode and
 * mxfa_cp_merge_launch as above.  local_buf: this rank's exchange buffer
 * (the entry `rank` of peer_bufs, as a host-side pointer). */
int mxfa_cp_attention_launch(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                             const int32_t* seqlens, void* out, float* lse, void* workspace, size_t workspace_bytes,
                             unsigned int* counters, const unsigned long long* peer_bufs, void* local_buf, int rank,
                             int world, int B, int HQ, int HKV, int D, int PS, int BTW, int num_pages, int num_splits,
                             int chunk_len, int bf16, float scale, void* stream);
/* 1 when the calling thread's last mxfa_cp_attention_launch merged inside the
 * decode kernel (one launch), 0 when it also launched the merge kernel. */
int mxfa_cp_last_merged_in_place(void);

/* Allocation-free variant of mxfa_kvcache_attention_launch.  It has no
 * counterpart in the reference.  It exists for callers that cannot allocate
 * device memory when they run attention (an engine that pre-reserved all GPU
 * memory for its own pools, a foreign-language host without a device
 * allocator, a latency-critical loop that must not risk the device sync a
 * cudaMalloc can cause).  Arguments match mxfa_kvcache_attention_launch
 * minus the workspace: the split partials go to one buffer of
 * MXFA_NOALLOC_SCRATCH_BYTES compiled into the library, which every GPU that
 * loads the library holds until the process exits.  Calls needing more
 * scratch than that fail with MXFA_ERR_UNSUPPORTED and a message (argument
 * errors are reported first, as by mxfa_kvcache_attention_launch).  The
 * first call on a device looks up the buffer's device address with that
 * device current (make that first call before any stream capture); a call
 * made after the device's context was re-created, as by cudaDeviceReset,
 * looks it up again.  All
 * calls on a device share the one buffer, so calls that overlap on the GPU
 * (other streams, other host threads) race and must be serialised by the
 * caller.  Nothing is allocated or freed by this call. */
#define MXFA_NOALLOC_SCRATCH_BYTES (4u << 20)
int mxfa_kvcache_attention_noalloc_launch(const void* q, const void* k_cache, const void* v_cache,
                                          const int32_t* block_table, const int32_t* seqlens, void* out,
                                          float* lse, int B, int Sq, int HQ, int HKV, int D, int PS, int BTW,
                                          int num_pages, int append_len, int num_splits, int chunk_len,
                                          int causal, int bf16, float scale, void* stream);

/* LSE merge of split partials (the reference's split_combine,
 * csrc_native/m1_kernel.cpp:862-888, generalised to strided partials).
 * Partial p of row r lives at ows[r*NP*D + p*D] and mdws[(r*NP + p)*2].
 * Writes out [rows, D] in bf16/fp16 when `out` != NULL, f32 [rows, D] when
 * `out_f32` != NULL, and the natural-log LSE [rows] when `lse` != NULL. */
int mxfa_split_combine_launch(const float* ows, const float* mdws, void* out, float* out_f32,
                              float* lse, int rows, int D, int NP, int bf16, void* stream);

/* Context-split decode, local half (no reference counterpart: the reference
 * is single-device).  Single-token attention of q [B, 1, HQ, D] over this
 * rank's positions of every sequence (its own pages, lengths and table),
 * written as packed f32 [B*HQ, D + 1]: the normalised O of each row followed
 * by its natural-log LSE (-inf, with O = 0, for a row with no local keys).
 * That packed buffer is what the ranks all-gather before
 * mxfa_lse_merge_launch.  Needs a split workspace of
 * mxfa_split_workspace_bytes(B*HQ, D, num_splits) bytes (num_splits 0 =
 * library plan, which then needs the plan's size). */
int mxfa_kvcache_attention_packed_launch(const void* q, const void* k_cache, const void* v_cache,
                                         const int32_t* block_table, const int32_t* seqlens, float* packed,
                                         void* workspace, size_t workspace_bytes, int B, int HQ, int HKV,
                                         int D, int PS, int BTW, int num_pages, int num_splits, int chunk_len,
                                         int bf16, float scale, void* stream);

/* Merge of per-rank (O, LSE) results for context-split decode across GPUs
 * (no reference counterpart: the reference is single-device).  `packed` is
 * f32 [N, rows, D + 1]: normalised O then the natural-log LSE of each row on
 * each of N ranks (the buffer an all-gather produces).  Writes the merged
 * out [rows, D] (bf16/fp16) and, if non-NULL, lse [rows]. */
int mxfa_lse_merge_launch(const float* packed, void* out, float* lse, int N, int rows, int D,
                          int bf16, void* stream);

/* ------------------------------------------------------------------ append */

/* Paged / dense KV append (reference.py:108-122): token i of sequence b
 * goes to logical position seqlens[b] + i, i.e. page
 * block_table[b, pos / PS], slot pos % PS (dense: row pos of cache b).
 * Bit-exact copy.  Does not change seqlens (see mxfa_seqlens_add_launch).
 *   k_new, v_new [B, Sk, HKV, D]; caches as in mxfa_kvcache_attention_launch.
 * Out-of-range pages / capacity are skipped and flagged, never written. */
int mxfa_kv_append_launch(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                          const int32_t* block_table, const int32_t* seqlens, int B, int Sk, int HKV,
                          int D, int PS, int BTW, int num_pages, int elem_bytes, void* stream);

/* seqlens[b] += delta on the device for int32 (is_int64 = 0) or int64
 * lengths -- the in-place `cache_seqlens.add_(k.shape[1])` of
 * reference.py:137-138 / dispatch.py:117-121, without a host sync. */
int mxfa_seqlens_add_launch(void* seqlens, int is_int64, int B, int delta, void* stream);

/* ----------------------------------------------------------------- prefill */

/* Causal / non-causal attention forward over packed variable-length
 * sequences: flash_attn_varlen_func (api.py:69-148, reference.py:60-85) and,
 * with cu_q == cu_k == NULL, the dense flash_attn_func (api.py:34-66) with
 * uniform lengths max_q / max_k per batch item.
 *   q [Tq, HQ, D], k/v [Tk, HKV, D] (dense: [B, max_q|max_k, H, D])
 *   cu_q, cu_k int32 [B + 1] device arrays (or NULL for dense)
 *   out [Tq, HQ, D]; lse optional f32 [Tq, HQ]
 *   total_q = Tq, total_k = Tk: the row counts of q and k/v (dense: B*max_q, B*max_k)
 * max_q must bound every q length (it sizes the grid).  Runs on the tcgen05
 * tensor cores (sm_100a), operands staged by TMA, accumulators in TMEM. */
int mxfa_varlen_fwd_launch(const void* q, const void* k, const void* v, const int32_t* cu_q,
                           const int32_t* cu_k, void* out, float* lse, int B, int max_q, int max_k,
                           int total_q, int total_k, int HQ, int HKV, int D, int causal, int bf16,
                           float scale, void* stream);

/* mxfa_varlen_fwd_launch with P kept at ~16 significant bits in the P.V
 * product: P is split into its value rounded to the input type and the
 * rounded remainder, and both are multiplied with V (1.5x the tensor work).
 * The default entry rounds P once to the input type, as FlashAttention
 * does; its error is at most u * (softmax-weighted mean of |V|), u = 2^-9
 * (bf16) or 2^-11 (fp16), which matters only when V has a wide dynamic
 * range.  No reference counterpart: the reference's fp32 CPU path
 * (reference.py:60-85) never rounds P. */
int mxfa_varlen_fwd_exact_launch(const void* q, const void* k, const void* v, const int32_t* cu_q,
                                 const int32_t* cu_k, void* out, float* lse, int B, int max_q, int max_k,
                                 int total_q, int total_k, int HQ, int HKV, int D, int causal, int bf16,
                                 float scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MXFA_B200_H_ */
