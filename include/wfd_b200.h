/*
 * wfd_b200.h — C ABI of the B200 wavefront-decoding attention / KV-slot library.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t (passed
 * as void*), launches asynchronously on that stream and returns an int status
 * (WFD_OK = 0).  Argument checks that need no device data are done on the host
 * and reported as a status before anything launches.  Checks that need device
 * data (slot ids, positions, cu_seqlens) are done inside the kernels, which skip
 * the offending work item and OR an error bit into the caller's device error
 * word `d_err` (int32, may be NULL); read it with wfd_read_error().  No kernel
 * traps, asserts or waits without a bound.
 *
 * Layouts (row-major, contiguous, the reference's own layouts):
 *   q, out            (n_rows, Hq, Dh)
 *   k_new, v_new      (n_rows, Hkv, Dh)               new K/V rows, row i <-> q row i
 *   k_cache, v_cache  (n_slots, n_seqs, max_seq, Hkv, Dh)
 *                     == BatchStaticKVCache.K / .V, buffer index == absolute position
 *                     (reference src/decoding/batch_kv_cache.py:28-44)
 *   lens              (n_slots, n_seqs) int32, logical slot lengths
 *                     == BatchStaticKVCache.seqlen (batch_kv_cache.py:44)
 *   packed k, v       (total_k, Hkv, Dh) with cu_k (n_seg+1) int32,
 *                     q (total_q, Hq, Dh) with cu_q (n_seg+1) int32
 *                     (reference fa4_attention.py:294-317)
 * dtype: WFD_DTYPE_BF16 or WFD_DTYPE_F32 (all tensors of one call share it).
 * GQA: query head hq reads kv head hq / (Hq / Hkv), as SDPA enable_gqa does.
 * Softmax statistics are accumulated in fp32 in every variant.
 */
#ifndef WFD_B200_H
#define WFD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Raised whenever a declaration or a struct layout below changes incompatibly
 * (2: wfd_sched_params.depth_slots; 3: wfd_commit_window takes n_rows;
 * 4: wfd_sched_params.gap_windows; 5: wfd_linear; 6: wfd_rope_split_norm,
 * wfd_silu_mul_norm). */
#define WFD_ABI_VERSION 6

enum wfd_status {
  WFD_OK = 0,
  WFD_ERR_INVALID_ARG = 1,     /* host-side argument check failed            */
  WFD_ERR_UNSUPPORTED = 2,     /* dtype / head_dim / GQA shape not built     */
  WFD_ERR_WORKSPACE = 3,       /* workspace missing or too small             */
  WFD_ERR_CUDA = 4,            /* a CUDA runtime call failed                 */
  WFD_ERR_ALIGNMENT = 5,       /* a pointer is not 16-byte aligned           */
  WFD_ERR_DEVICE_TIMEOUT = 16, /* device error word: bounded wait gave up    */
  WFD_ERR_DEVICE_BOUNDS = 17   /* device error word: index/length out of range */
};

enum wfd_dtype { WFD_DTYPE_BF16 = 0, WFD_DTYPE_F32 = 1 };

/* One wavefront work item: q_len query rows of sequence `seq` that sit at
 * absolute positions pos0 .. pos0+q_len-1 of KV slot `slot`.  Row j of the item
 * (q / k_new row q_row0 + j) writes its K/V at position pos0 + j and attends
 * keys [0, pos0 + j] of that slot (bottom-right causal inside the window).
 * q_len == 1 is the wavefront decode row; q_len > 1 is a verify window or a
 * group of rows sharing one slot.  Mirrors the (slots, seq_ids, positions)
 * triples of BatchStaticKVCache.write_tokens / gather_pack
 * (batch_kv_cache.py:61-96) and the grouped segments of
 * OuroBlocksBatch.advance_union (ouro_blocks_batch.py:180-231). */
typedef struct wfd_item {
  int32_t slot;
  int32_t seq;
  int32_t pos0;
  int32_t q_len;
  int32_t q_row0;
} wfd_item;

/* Library identity. */
int wfd_abi_version(void);
const char* wfd_status_string(int status);

/* Copy the device error word to *h_err and reset it to 0 (synchronises
 * `stream`).  Returns WFD_OK, or WFD_ERR_DEVICE_TIMEOUT / _BOUNDS when the word
 * was non-zero.  Bits: 1 bounded wait gave up, 2 slot / sequence out of range,
 * 4 position or length past the slot capacity, 8 row index outside the given
 * tensors, 16 bad cu_seqlens, 128 a device-scheduler invariant (token-slot
 * overflow, two commit points of one sequence in a tick, R union over capacity). */
int wfd_read_error(int32_t* d_err, int32_t* h_err, void* stream);

/* Batch-invariant attention (process-wide, default off).  On: bf16 attention runs
 * on the tensor-core kernel with every (item, kv head) unit processed whole by
 * one CTA — no split, no merge — so a row's output depends on its own unit
 * only, not on the other items of the launch (what bit-exact greedy equality of
 * wavefront and sequential decoding needs, together with fixed GEMM shapes).
 * Read when a launch is built: a captured CUDA graph keeps its mode.  fp32 stays
 * on the CUDA-core kernel, which is not batch-invariant.  No counterpart in the
 * reference. */
int wfd_set_batch_invariant(int32_t on);
int wfd_get_batch_invariant(void);

/* Test hook (process-wide, default off): on != 0 makes every CTA of the tcgen05
 * attention kernel give up right after issuing its first K/V copies, as it does
 * when a bounded mbarrier wait runs out (2^20 polls, a multi-second ceiling):
 * bit 1 of the error word is set (WFD_ERR_DEVICE_TIMEOUT from wfd_read_error),
 * the CTA stops issuing copies and MMAs, waits (with the normal bound) for the
 * ones in flight, frees its tensor memory and returns; outputs are undefined.
 * Read when a launch is built.  No counterpart in the reference. */
int wfd_test_fail_waits(int32_t on);

/* Bytes of device workspace the attention entry points need for up to
 * `max_items` work items / segments.  The workspace must be zero-filled once
 * after allocation (wfd_workspace_init); the kernels leave it zeroed again. */
size_t wfd_workspace_bytes(int32_t max_items, int32_t head_dim, int32_t dtype);
int wfd_workspace_init(void* workspace, size_t bytes, void* stream);

/* Wavefront decode / verify attention over KV slots, with the K/V append fused.
 *
 * Replaces, per reference call site, the sequence
 *   BatchStaticKVCache.write_tokens   (batch_kv_cache.py:61-73)
 *   BatchStaticKVCache.gather_pack    (batch_kv_cache.py:75-96)
 *   fa4_attention.attn_varlen / attn_varlen_q1_padded (fa4_attention.py:301-342)
 * made by OuroBlocksBatch.advance_union (ouro_blocks_batch.py:207-231) and
 * HuginnBlocksBatch._union_attn (huginn_blocks_batch.py:254-285), and the
 * per-row graph-engine loop of `_fa_varlen` + index_copy_
 * (graph_blocks.py:171-194, 306-328).
 *
 * For every item: writes k_new/v_new rows into the cache at (slot+slot_offset,
 * seq, pos0+j), raises lens[slot+slot_offset][seq] to at least pos0+q_len (if
 * lens != NULL), and writes out rows q_row0.. with the attention of each row
 * over its slot prefix.  Keys in [0, pos0) are read in place from the cache;
 * the window keys come from k_new/v_new.  `slot_offset` lets one item table
 * serve every layer of a tick (slot = depth * n_layers + layer in the
 * reference, ouro_blocks_batch.py:77-78).  `items` is a DEVICE array so the
 * table can be updated between CUDA-graph replays.  scale <= 0 selects
 * 1/sqrt(head_dim).  Chooses the CUDA-core decode kernel or the tcgen05 verify
 * kernel from max_q (largest q_len in the table; an upper bound is fine). */
int wfd_wave_attn(const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                  void* out, int32_t* lens, const wfd_item* items, int32_t n_items, int32_t max_q,
                  int32_t slot_offset, int32_t n_rows, int32_t n_slots, int32_t n_seqs, int32_t max_seq,
                  int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype, float scale,
                  void* workspace, size_t workspace_bytes, int32_t* d_err, void* stream);

/* wfd_wave_attn without a caller-supplied workspace, for callers that cannot
 * allocate device memory when they call: serving runtimes that fix their
 * memory plan at start-up and must not allocate per request (an allocation can
 * synchronise the device or fail under memory pressure mid-request), and
 * foreign-language hosts that hold raw device pointers but have no device
 * allocator of their own.  Has no counterpart in the reference.
 *
 * The scratch memory is a fixed array inside the library (5.5 MB on every
 * device that loads the library, held until the process exits).  Limits:
 * bf16 tensors, head_dim 128 (the tcgen05 kernel), at most 4096 items, at
 * most 160 SMs, fewer than 2^31 cache rows; anything else returns
 * WFD_ERR_UNSUPPORTED or WFD_ERR_WORKSPACE, and every host-side argument check
 * runs before anything is queued on the stream.  The first call on a device,
 * whatever its arguments, looks up the array's device address (once per
 * device, with that device current), so make that first call before any
 * stream capture.  Every call shares the one array: each call clears the part
 * that must start at zero, but calls that overlap on the GPU (different
 * streams, or different threads racing on one stream) corrupt each other's
 * results.  Allocates nothing: no cudaMalloc, no allocating library routine.
 * Arguments as wfd_wave_attn. */
int wfd_wave_attn_static(const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                         void* out, int32_t* lens, const wfd_item* items, int32_t n_items, int32_t max_q,
                         int32_t slot_offset, int32_t n_rows, int32_t n_slots, int32_t n_seqs, int32_t max_seq,
                         int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype, float scale,
                         int32_t* d_err, void* stream);

/* Same as wfd_wave_attn but forces the kernel: 0 = CUDA-core decode kernel,
 * 1 = tcgen05 verify kernel.  For tests and benchmarks. */
int wfd_wave_attn_kernel(int32_t which, const void* q, const void* k_new, const void* v_new, void* k_cache,
                         void* v_cache, void* out, int32_t* lens, const wfd_item* items, int32_t n_items,
                         int32_t max_q, int32_t slot_offset, int32_t n_rows, int32_t n_slots, int32_t n_seqs,
                         int32_t max_seq, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype,
                         float scale, void* workspace, size_t workspace_bytes, int32_t* d_err, void* stream);

/* wfd_wave_attn with the kernel choice of wfd_wave_attn_kernel (-1 auto) and
 * optional per-row positions: row j of item i sits at position
 * row_pos[(q_row0 + j) * row_pos_stride] (increasing within the item, the first
 * one equal to pos0) instead of pos0 + j, is appended there and attends keys
 * [0, that position] of its slot.  This is a gapped window: the reference
 * pads such runs (the tokens of one sequence on one depth slot under KV
 * sharing, ouro_blocks_batch.py:184-205) into one zero-padded span; here the
 * rows keep their own positions and the prefix is still read once per window.
 * row_pos == NULL is wfd_wave_attn.  Gapped windows run on the tcgen05 kernel
 * only (bf16, head_dim 64 / 128); otherwise WFD_ERR_UNSUPPORTED.  A middle row
 * whose position is out of order is skipped and reported in the error word. */
int wfd_wave_attn_rows(int32_t which, const void* q, const void* k_new, const void* v_new, void* k_cache,
                       void* v_cache, void* out, int32_t* lens, const wfd_item* items, int32_t n_items, int32_t max_q,
                       const int32_t* row_pos, int32_t row_pos_stride, int32_t slot_offset, int32_t n_rows,
                       int32_t n_slots, int32_t n_seqs, int32_t max_seq, int32_t n_heads, int32_t n_kv_heads,
                       int32_t head_dim, int32_t dtype, float scale, void* workspace, size_t workspace_bytes,
                       int32_t* d_err, void* stream);

/* Packed varlen attention, drop-in for fa4_attention.attn_varlen
 * (fa4_attention.py:301-317) and for the graph engine's direct
 * aten._flash_attention_forward call (graph_blocks.py:37-43).  Segment i: query
 * rows [cu_q[i], cu_q[i+1]), key rows [cu_k[i], cu_k[i+1]) of k / v.
 * causal != 0: bottom-right causal per segment (row r sees keys
 * <= k_len - q_len + r); causal == 0: every row sees the whole segment.
 * cu_q / cu_k are DEVICE int32 arrays (lengths as data, graph_blocks.py:5-11).
 * total_k bounds the key rows any cu_k entry may address. */
int wfd_attn_varlen(const void* q, const void* k, const void* v, void* out, const int32_t* cu_q,
                    const int32_t* cu_k, int32_t n_seg, int32_t max_q, int32_t total_q, int32_t total_k,
                    int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype, int32_t causal,
                    float scale, void* workspace, size_t workspace_bytes, int32_t* d_err, void* stream);

/* Explicit-segment attention: segment i has query rows [q_row0[i], +q_len[i])
 * and key rows [k_row0[i], +k_len[i]), bottom-right causal when causal != 0.
 * Segments may share key rows.  Serves attn_dense (fa4_attention.py:191-232)
 * and attn_cutoff_multi (fa4_attention.py:240-291) where each query has its
 * own key cutoff.  All arrays are DEVICE int32. */
int wfd_attn_segments(const void* q, const void* k, const void* v, void* out, const int32_t* q_row0,
                      const int32_t* q_len, const int32_t* k_row0, const int32_t* k_len, int32_t n_seg,
                      int32_t max_q, int32_t total_q, int32_t total_k, int32_t n_heads, int32_t n_kv_heads,
                      int32_t head_dim, int32_t dtype, int32_t causal, float scale, void* workspace,
                      size_t workspace_bytes, int32_t* d_err, void* stream);

/* KV append: BatchStaticKVCache.write_tokens (batch_kv_cache.py:61-73).  Row i
 * of k_new / v_new goes to (slots[i]+slot_offset, seqs[i], positions[i]);
 * lens[slot][seq] = max(lens, positions[i] + 1) when lens != NULL.  Device int32
 * index arrays.  Out-of-range rows are skipped and flagged (the reference
 * raises IndexError, batch_kv_cache.py:70-71). */
int wfd_append(const void* k_new, const void* v_new, void* k_cache, void* v_cache, int32_t* lens,
               const int32_t* slots, const int32_t* seqs, const int32_t* positions, int32_t n, int32_t slot_offset,
               int32_t n_slots, int32_t n_seqs, int32_t max_seq, int32_t n_kv_heads, int32_t head_dim,
               int32_t dtype, int32_t* d_err, void* stream);

/* Prefill write: BatchStaticKVCache.write_prefill (batch_kv_cache.py:51-59).
 * k, v (n_seqs, L, Hkv, Dh) go to positions [0, L) of `slot` for every
 * sequence; lens[slot][*] = max(lens, L). */
int wfd_write_prefill(const void* k, const void* v, void* k_cache, void* v_cache, int32_t* lens, int32_t slot,
                      int32_t L, int32_t n_slots, int32_t n_seqs, int32_t max_seq, int32_t n_kv_heads,
                      int32_t head_dim, int32_t dtype, void* stream);

/* Rollback commit: BatchStaticKVCache.drop_positions_at_and_after
 * (batch_kv_cache.py:99-105) for many sequences at once.  For every sequence b
 * with drop_pos[b] >= 0: lens[s][b] = min(lens[s][b], drop_pos[b]) for all
 * slots s.  K/V buffers are untouched (stale tails are never read). */
int wfd_commit_drop(int32_t* lens, const int32_t* drop_pos, int32_t n_slots, int32_t n_seqs, void* stream);

/* Accept commit for verify windows.  For item i (slot, seq, pos0, q_len,
 * q_row0) the accepted rows are either rows [0, accept_len[i]) (accept_len !=
 * NULL, the greedy accept-prefix of the DtV cascade, scheduler_batch.py:472-499)
 * or the rows whose accept_mask byte (indexed by q row) is non-zero.  Accepted
 * rows are compacted in place to positions pos0, pos0+1, ... of the slot (a
 * no-op when they already form a prefix), lens[slot+slot_offset][seq] is set to
 * pos0 + n_accepted, acc_rows[q_row0 + k] receives the q row of the k-th
 * accepted row and acc_count[i] the count (either output may be NULL).
 * n_rows: entries of accept_mask / acc_rows (q rows); an item whose window rows
 * fall outside [0, n_rows) is skipped and reported in the error word. */
int wfd_commit_window(void* k_cache, void* v_cache, int32_t* lens, const wfd_item* items, int32_t n_items,
                      const int32_t* accept_len, const uint8_t* accept_mask, int32_t* acc_rows,
                      int32_t* acc_count, int32_t n_rows, int32_t slot_offset, int32_t n_slots, int32_t n_seqs,
                      int32_t max_seq, int32_t n_kv_heads, int32_t head_dim, int32_t dtype, int32_t* d_err,
                      void* stream);

/* Dense prompt attention over n_seqs segments of equal lengths (the prompt pass,
 * write_prefill + attn_dense of the reference, ouro_blocks_batch.py:123-144,
 * fa4_attention.py:191-232): q (n_seqs * q_len, Hq, Dh), k / v (n_seqs * k_len,
 * Hkv, Dh), out like q.  causal != 0: bottom-right causal per segment (row i
 * sees keys j <= i + k_len - q_len; q_len == k_len is the ordinary causal
 * mask), else every row sees its whole segment.  bf16, head_dim 64 or 128 (the
 * tcgen05 prompt kernel); other dtypes / head dims return WFD_ERR_UNSUPPORTED.
 * scale <= 0 selects 1/sqrt(head_dim).  Rows that see no key get zeros. */
int wfd_attn_prefill(const void* q, const void* k, const void* v, void* out, int32_t n_seqs, int32_t q_len,
                     int32_t k_len, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype,
                     int32_t causal, float scale, int32_t* d_err, void* stream);

/* Gather packed prefixes, BatchStaticKVCache.gather_pack (batch_kv_cache.py:75-96):
 * segment i copies positions [0, uptos[i]] of (slots[i], seqs[i]) into rows
 * cu_k[i] .. of k_pack / v_pack.  cu_k (n+1) is a DEVICE int32 array the caller
 * computed (cu_k[i+1] - cu_k[i] == uptos[i] + 1).  Kept for API parity; the
 * wavefront kernels read slots in place and never need it. */
int wfd_gather_pack(const void* k_cache, const void* v_cache, void* k_pack, void* v_pack, const int32_t* slots,
                    const int32_t* seqs, const int32_t* cu_k, int32_t n, int32_t n_slots, int32_t n_seqs,
                    int32_t max_seq, int32_t n_kv_heads, int32_t head_dim, int32_t dtype, int32_t* d_err,
                    void* stream);

/* ---------------------------------------------------------------------------
 * Looped-LM block helpers used by the wavefront engine around the attention
 * (fused element-wise work of one transformer block; fp32 arithmetic, bf16 or
 * f32 storage).  The reference runs these as framework modules (norm, RoPE in
 * fa4_attention.compute_qkv, fa4_attention.py:140-160, the SwiGLU MLP), so they
 * have no C counterpart in it.
 * ------------------------------------------------------------------------- */

/* RMSNorm: y[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w for n rows of d
 * (d % 8 == 0; x, w, y 16-byte aligned; y does not overlap x). */
int wfd_rmsnorm(const void* x, const void* w, void* y, int32_t n, int32_t d, float eps, int32_t dtype,
                void* stream);

/* Split a fused QKV projection qkv (n, (H + 2 Hkv) * Dh) into q (n, H, Dh),
 * k (n, Hkv, Dh) rotated by RoPE and v (n, Hkv, Dh).  style 0 rotates dims
 * (i, i + Dh/2), style 1 dims (2i, 2i + 1), by angle pos * theta_i with cos / sin
 * tables (max_pos, Dh/2) fp32.  Row r's position is pos[r * pos_stride] (device
 * int32), or r % pos_period when pos is NULL.  A position outside [0, max_pos)
 * sets the bad-position bit of the device error word d_err (wfd_read_error)
 * and uses position 0. */
int wfd_rope_split(const void* qkv, const float* cos_tab, const float* sin_tab, const int32_t* pos,
                   int32_t pos_stride, int32_t pos_period, int32_t max_pos, void* q, void* k, void* v, int32_t n,
                   int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t style, int32_t dtype,
                   int32_t* d_err, void* stream);

/* SwiGLU gate: out (n, dff) = silu(g) * u where gu (n, 2 dff) = [g | u] per row
 * (dff % 8 == 0). */
int wfd_silu_mul(const void* gu, void* out, int32_t n, int32_t dff, int32_t dtype, void* stream);

/* RMSNorm folded into the next linear layer.  With W' = diag(norm weight) W the
 * projection of the normalised row is s_r * (x_r . W'), s_r = rsqrt(mean(x_r^2) +
 * eps); the GEMM takes x itself and these variants apply s_r to its output:
 * wfd_rope_split_norm is wfd_rope_split of s_r * qkv_r (v included);
 * wfd_silu_mul_norm is out = silu(s_r g) * (s_r u).  x: (n, d) with row stride ldx
 * elements, the rows the GEMM read (d % 8 == 0, ldx % 8 == 0, 16-byte aligned).  Each
 * row is processed independently of the others. */
int wfd_rope_split_norm(const void* qkv, const void* x, int32_t ldx, int32_t d, float eps, const float* cos_tab,
                        const float* sin_tab, const int32_t* pos, int32_t pos_stride, int32_t pos_period,
                        int32_t max_pos, void* q, void* k, void* v, int32_t n, int32_t n_heads, int32_t n_kv_heads,
                        int32_t head_dim, int32_t style, int32_t dtype, int32_t* d_err, void* stream);
int wfd_silu_mul_norm(const void* gu, const void* x, int32_t ldx, int32_t d, float eps, void* out, int32_t n,
                      int32_t dff, int32_t dtype, void* stream);

/* Linear layer of a few rows on the tensor cores with the block's element-wise
 * work fused in (bf16; fp32 accumulation).  y = s_r * x_r . W for W (K, F)
 * row-major, where s_r = rsqrt(mean(x_r^2) + eps) when row_norm is set (an
 * RMSNorm whose weight the caller has multiplied into W's rows) and 1 otherwise;
 * then, by mode:
 *   WFD_LINEAR_PLAIN     out (n_rows, F) = y
 *   WFD_LINEAR_RESIDUAL  out (n_rows, F) += y, in place
 *   WFD_LINEAR_SWIGLU    W's columns interleave gate and up projections per 64
 *                        (columns 128j.. = gate features 64j..64j+63, then the up
 *                        features 64j..): out (n_rows, F / 2) = silu(g) * u, with g
 *                        and u rounded to bf16 first (F % 128 == 0)
 *   WFD_LINEAR_ROPE      F = (H + 2 Hkv) Dh (F % 128 == 0, Dh 64 or 128): y rounded to
 *                        bf16, then split and rotated as wfd_rope_split does
 * The reference runs these as framework modules around its attention backend
 * (RMSNorm, q/k/v/o projections, RoPE, SwiGLU MLP; ouro_blocks_batch.py:100-121),
 * so this has no C counterpart in it.  Rows are processed independently of each
 * other: a row's result does not depend on n_rows.  x, w, out, q, k, v 16-byte
 * aligned; K % 8 == 0, ldx % 8 == 0, ldx >= K. */
enum wfd_linear_mode { WFD_LINEAR_PLAIN = 0, WFD_LINEAR_RESIDUAL = 1, WFD_LINEAR_SWIGLU = 2, WFD_LINEAR_ROPE = 3 };

typedef struct wfd_linear_params {
  const void* x;            /* (n_rows, K) bf16 rows, row stride ldx elements          */
  const void* w;            /* (K, F) bf16, row-major                                    */
  void* out;                /* plain / residual: row stride ldo; swiglu: (n_rows, F / 2) */
  void* q;                  /* rope: q (n_rows, H, Dh), k / v (n_rows, Hkv, Dh)         */
  void* k;
  void* v;
  const float* cos_tab;     /* rope: (max_pos, Dh / 2) fp32                              */
  const float* sin_tab;
  const int32_t* pos;       /* rope: row r at pos[r * pos_stride]; NULL: r % pos_period  */
  int32_t* err;             /* device error word (wfd_read_error)                        */
  int32_t n_rows, K, F, ldx, ldo;
  int32_t mode, row_norm;
  float eps;
  int32_t H, Hkv, Dh, rope_style, pos_stride, pos_period, max_pos;
} wfd_linear_params;

int wfd_linear(const wfd_linear_params* p, void* stream);
/* sizeof(wfd_linear_params) as compiled into the library. */
size_t wfd_linear_params_bytes(void);

/* Row gather: out[i] = a[idx[i * idx_stride]] (+ b[same row] when b != NULL),
 * rows of d elements (d % 8 == 0), n_src rows in a / b.  An index outside
 * [0, n_src) sets the bad-rows bit of d_err and reads row 0. */
int wfd_gather_rows(const void* a, const void* b, const int32_t* idx, int32_t idx_stride, void* out, int32_t n,
                    int32_t d, int32_t n_src, int32_t dtype, int32_t* d_err, void* stream);

/* Row scatter: dst[idx[i * idx_stride]] = src[i], and zero[that row] = 0 when
 * zero != NULL; an index outside [0, n_dst) sets the bad-rows bit and is skipped. */
int wfd_scatter_rows(const void* src, const int32_t* idx, int32_t idx_stride, void* dst, void* zero, int32_t n,
                     int32_t d, int32_t n_dst, int32_t dtype, int32_t* d_err, void* stream);

/* Wave item table from a union table of int32 rows of `cols` columns:
 * items[i] = {tab[i][c_slot], tab[i][c_seq], tab[i][c_pos], tab[i][c_qlen], i}. */
int wfd_items_from_table(const int32_t* tab, int32_t cols, int32_t c_slot, int32_t c_seq, int32_t c_pos,
                         int32_t c_qlen, wfd_item* items, int32_t n, void* stream);

/* Greedy ids: out[r] = the first index of the maximum of logits row r (n rows of V). */
int wfd_argmax_rows(const void* x, int32_t* out, int32_t n, int32_t V, int32_t dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Device-side wavefront scheduling (route / settle of scheduler_batch.py:268-360
 * as kernels, so one CUDA graph runs a whole tick; no counterpart in the
 * reference, whose scheduler runs on the host with one read-back per tick).
 * Token slot j of sequence b is entry b * W + j of the slot arrays and pool row
 * b * W + j of the engine.  State: 0 free, 1 queued for the prelude, 2 in the
 * wave.  Tables use the engine's int32 union-row layout (pool row, position,
 * token, cache sequence, slot base, live, per-layer first cache rows).
 * ------------------------------------------------------------------------- */
typedef struct {
  int32_t *alive, *state, *tok, *pos, *step;     /* token slots (B * W) */
  int32_t *n_commit, *done, *committed, *seq_ct; /* (B), (B), (B, max_new), (B, 8) */
  const uint8_t* emu;                            /* (B, emu_len) accept draws, NULL = greedy */
  int32_t *emu_ctr, *batch_ct;                   /* (B), (8) */
  unsigned long long* keys;                      /* (3) sum of k_len over P / R / C rows */
  int32_t *c_slot, *lens, *err;                  /* (2B), KV lengths (n_kv_slots, lens_stride), error word */
  int32_t *p_tab, *r_tab, *c_tab;                /* (B, p_cols), (r_cap, 6), (2B, c_cols) */
  const int32_t* c_out;                          /* (2B) greedy ids of the C union */
  int32_t B, W, T_total, T_draft, max_new, emu_len;
  int32_t n_core, n_kv_slots, lens_stride, max_seq;
  int32_t p_cols, c_cols, r_cap;
  int32_t scratch_row, scratch_seq;
  int32_t p_slot0, n_prelude, c_slot0, n_coda;
  int32_t depth_slots; /* core depth slots: T_total, or the KV-sharing budget s (depth r -> slot r % s) */
  int32_t gap_windows; /* 1: all of a sequence's tokens on one depth slot form one R window, gaps included
                          (attended with per-row positions); 0: only runs of consecutive positions do */
} wfd_sched_params;

/* sizeof(wfd_sched_params) as compiled into the library: a host that mirrors the
 * struct (ctypes, cgo, JNI) checks its layout against it. */
size_t wfd_sched_params_bytes(void);

/* Before the P union: queue -> wave for each sequence's queued token (P table
 * row b), compacted R table of every live token.  B <= 1024, W <= 32. */
int wfd_sched_pre_tick(const wfd_sched_params* p, void* stream);
/* After the R union: advance steps, route commit points (C row 2b) and draft
 * points (C row 2b + 1). */
int wfd_sched_route(const wfd_sched_params* p, void* stream);
/* After the C union: accept / reject the successor of each commit point,
 * cascade rollback (KV lengths truncated), queue the next token and the new
 * leading-edge draft, commit tokens and per-sequence counters. */
int wfd_sched_settle(const wfd_sched_params* p, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WFD_B200_H */
