/*
 * hcu_indexer.h -- C ABI of the B200 (sm_100a) DSA lightning-indexer library
 * (libhcu_indexer.so).
 *
 * Plain pointers, sizes and a CUDA stream; no torch types.  Every entry point
 * only enqueues work on `stream` (no host synchronisation, no allocation), so
 * every call is CUDA-graph capturable.  Outputs and workspaces are owned by the
 * caller; `*_workspace_bytes` queries size them.  Launch configuration depends
 * only on the static shapes passed here and the device's SM count.
 *
 * Return value: HCU_OK or an error code; nothing throws across this ABI.
 * HCU_ERR_ARG          an argument violates the contract (nothing launched)
 * HCU_ERR_UNSUPPORTED  a shape/option this build does not implement
 * HCU_ERR_LAUNCH       the CUDA launch failed (cudaGetLastError != success)
 * Device-side faults that must not hang the GPU (a bounded wait that expired)
 * are recorded in a sticky device status word read by hcu_read_device_status().
 *
 * Reference interface: the pybind11 module `hcu_ops._C`
 * (hcu_ops/csrc/bind.cpp:3-10,36-44,47-51,76-80 of charliedhw/sglang0.5.18-opt)
 * and the Triton dequant of prefill/patches/patch_fast_dequant.py:80-98.
 */
#ifndef HCU_INDEXER_H_
#define HCU_INDEXER_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* hcu_stream_t; /* == cudaStream_t */

enum {
  HCU_OK = 0,
  HCU_ERR_ARG = 1,
  HCU_ERR_LAUNCH = 2,
  HCU_ERR_TIMEOUT = 3,
  HCU_ERR_UNSUPPORTED = 4,
};

/* Element types of typed inputs. */
enum {
  HCU_DTYPE_F32 = 0,
  HCU_DTYPE_BF16 = 1,
};

/* Device status bits (sticky until cleared). */
enum {
  HCU_STATUS_WAIT_TIMEOUT = 1u << 0, /* an mbarrier / flag wait hit its bound */
  HCU_STATUS_BAD_INPUT = 1u << 1,    /* a kernel saw an out-of-range index and skipped it */
};

/* Sets the limit of every bounded wait of the library's kernels on the current
 * device (0 restores the default of 2 s).  A wait that reaches it records
 * HCU_STATUS_WAIT_TIMEOUT and the kernel returns without finishing its work, so
 * the context stays usable.  Synchronous; call it outside stream capture.  (No
 * counterpart in the reference, whose kernels wait without a bound.) */
int hcu_set_wait_limit_ns(uint64_t ns);

/* Library version string and the compile target ("sm_100a"). */
const char* hcu_version(void);

/* Reads (and with clear != 0 resets) the device status word of the current
 * device; synchronises the device.  Returns HCU_OK or HCU_ERR_LAUNCH. */
int hcu_read_device_status(uint32_t* status, int clear);

/* Last CUDA error string seen by this library on this thread ("" if none). */
const char* hcu_last_error_string(void);

/* ------------------------------------------------------------------------
 * Stage 1: paged K-cache dequant
 * ------------------------------------------------------------------------ */

/* MLA latent slot dequant, drop-in for sglang's dequantize_k_cache_paged with
 * the 656-byte slot (replaces prefill/patches/patch_fast_dequant.py:80-98 and
 * its kernel :45-70).
 *   quant_k_cache  uint8 [pool_slots, slot_stride] ; slot = 512 fp8 e4m3 |
 *                  4 fp32 group scales | 64 bf16 rope; slot_stride % 16 == 0
 *   page_table_1   int32 [n_tokens] slot index per output token
 *   out            bf16 [n_tokens, 576] (row stride 576 elements)
 * out[t, 128g+j] = bf16_rne(f32(fp8[s,128g+j]) * scale[s,g]); out[t,512:] = rope[s].
 * Slot indices outside [0, pool_slots) are skipped (output row untouched) and
 * flagged HCU_STATUS_BAD_INPUT. */
int hcu_dequant_k_cache_paged(const uint8_t* quant_k_cache, int64_t pool_slots, int64_t slot_stride,
                              const int32_t* page_table_1, int64_t n_tokens, uint16_t* out,
                              hcu_stream_t stream);

/* Indexer-K dequant (new in this build; the page layout of the logits op,
 * hcu_ops/csrc/mqa_hist.cu:77-91): page = 64 x 128 fp8 then 64 fp32 scales.
 *   kv_cache   uint8 [n_pages, page_stride] (page_stride >= 8448, % 16 == 0)
 *   token_loc  int32 [n_tokens] = page * 64 + offset
 *   out        bf16 [n_tokens, 128] */
int hcu_dequant_index_k_paged(const uint8_t* kv_cache, int64_t n_pages, int64_t page_stride,
                              const int32_t* token_loc, int64_t n_tokens, uint16_t* out,
                              hcu_stream_t stream);

/* MLA decode front end in one launch (replaces _C.rope_qout_kv_store,
 * hcu_ops/csrc/mla_kv.cu:183-240 / bind.cpp:32): for each of n_tokens tokens,
 *   q_out[t, h] = rope(q_pe[t, h]) for the nq heads (q_out may be q_pe itself);
 *   kv_c[t] = bf16((x * rstd) * w), rstd = rsqrt(sum(x^2) / 512 + norm_eps), in place
 *     (rsqrt_mode 2: 1 / sqrtf, IEEE; modes 0 and 1: rsqrtf);
 *   k_pe[t] = rope(k_pe[t]) in place;
 *   for t < n_loc, the 656-byte slot kv_buffer[loc[t]]: the fp8 e4m3 bytes of kv_c[t] in four
 *     128-element groups (scale = max(amax, store_eps) / 448, bytes of y * (1 / scale), round to
 *     nearest even, saturated), the four fp32 scales at +512, the rotated k_pe as bf16 at +528.
 * rope: bf16 [*, 64] with cos_sin_cache[pos] = 32 cos then 32 sin (bf16); pairs (2r, 2r+1), or
 * (r, 32 + r) with is_neox; every product and the difference / sum rounded to bf16.
 * All tensors bf16 except positions (int32, or int64 with positions_int64), loc (int64) and
 * kv_buffer (uint8); strides in elements.  kv_c rows and kv_weight 16-byte aligned
 * (kv_tok % 8 == 0); kv_buffer 16-byte aligned with slot_stride % 16 == 0, >= 656.  A position
 * outside [0, n_pos) skips its token, a slot outside [0, n_slots) is not written; both set
 * HCU_STATUS_BAD_INPUT. */
int hcu_rope_qout_kv_store(const void* positions, int32_t positions_int64, int64_t n_tokens, const uint16_t* q_pe,
                           int64_t nq, int64_t q_tok, int64_t q_head, uint16_t* q_out, int64_t qo_tok,
                           int64_t qo_head, uint16_t* kv_c, int64_t kv_tok, const uint16_t* kv_weight,
                           float norm_eps, uint16_t* k_pe, int64_t k_tok, const uint16_t* cos_sin_cache,
                           int64_t n_pos, int32_t is_neox, uint8_t* kv_buffer, int64_t n_slots,
                           int64_t slot_stride, const int64_t* loc, int64_t n_loc, float store_eps,
                           int32_t rsqrt_mode, hcu_stream_t stream);

/* Indexer-K cache writer (no counterpart among the reference's sources: sglang's
 * store is not vendored; this produces the page layout the logits op reads,
 * hcu_ops/csrc/mqa_hist.cu:77-91).  Per token: scale = max(amax, 1e-12) / 448,
 * fp8 e4m3 of x / scale (IEEE round-to-nearest division, saturating
 * round-to-nearest-even conversion); the 128 fp8 bytes go to page * page_stride
 * + offset * 128 and the scale to page * page_stride + 8192 + offset * 4.
 *   k          fp32 or bf16 (k_dtype) [n_tokens, k_stride >= 128 elements], 16-byte aligned rows;
 *              bf16 is widened to fp32 exactly before the arithmetic
 *   token_loc  int32 [n_tokens] = page * 64 + offset; out-of-range slots are
 *              skipped and flagged HCU_STATUS_BAD_INPUT; two tokens naming one
 *              slot race (one of them wins)
 *   kv_cache   uint8 [n_pages, page_stride] (page_stride >= 8448, % 16 == 0), written in place */
int hcu_quant_store_index_k_paged(const void* k, int32_t k_dtype, int64_t k_stride, const int32_t* token_loc,
                                  int64_t n_tokens, uint8_t* kv_cache, int64_t n_pages, int64_t page_stride,
                                  hcu_stream_t stream);

/* ------------------------------------------------------------------------
 * Stage 2: MQA index logits  s = (sum_h w[h] * relu(q_h . k)) * k_scale
 * ------------------------------------------------------------------------ */

/* Workspace (int32 elements) of the fused pass-1 histogram: rows * (2*4096+2). */
int64_t hcu_topk_hist_ws_elems(int64_t rows);

/* Paged decode logits; replaces _C.mqa_logits_hist (hcu_ops/csrc/mqa_hist.cu:324-405,
 * bind.cpp:41-44,78-80).
 *   q            fp8 e4m3 [batch, heads, 128] contiguous (heads 32 or 64)
 *   kv_cache     uint8 pages [n_pages, page_stride]
 *   weights      fp32 [batch, heads] (q scale folded in)
 *   context_lens int32 [batch]; clamped to [0, max_context_len]
 *   block_table  int32 [batch, bt_stride]; rows of a group of `group_size`
 *                share the table of the group's first row
 *   max_context_len == (block-table capacity) * 64 = logits row width
 *   logits       fp32 [batch, max_context_len]; written only where the mask bit is set
 *   mask         int16 [batch, max_context_len/16]; bit j of word i = token 16i+j
 *   hist_lens    optional int32 [batch]; when non-null also builds the top-k
 *                pass-1 workspace `zws` (int32 [hcu_topk_hist_ws_elems(batch)])
 *                for rows with min(hist_len, width) > 2048
 *   persistent_ctas / rows_per_cta: tuning hints of the reference API; <= 0 = auto */
int hcu_mqa_logits_hist(const uint8_t* q, int64_t batch, int64_t heads, const uint8_t* kv_cache,
                        int64_t n_pages, int64_t page_stride, const float* weights,
                        const int32_t* context_lens, const int32_t* block_table, int64_t bt_stride,
                        int64_t max_context_len, int64_t group_size, int64_t persistent_ctas,
                        int64_t rows_per_cta, const int32_t* hist_lens, float* logits, int16_t* mask,
                        int32_t* zws, hcu_stream_t stream);

/* Ragged prefill logits (new; the prefill indexer of the reference is closed
 * lightop _mqa_logits).  Query row r sees tokens [row_start[r], row_end[r]) of a
 * contiguous fp8 K; same logits + mask contract as hcu_mqa_logits_hist with the
 * row width = n_tokens.
 *   q        fp8 [rows, heads, 128]; weights fp32 [rows, heads]
 *   k_fp8    fp8 [n_tokens, 128]; k_scale fp32 [n_tokens]
 *   logits   fp32 [rows, logits_stride] (logits_stride >= n_tokens, % 4 == 0)
 *   mask     int16 [rows, logits_stride/16] */
int hcu_mqa_logits_ragged(const uint8_t* q, int64_t rows, int64_t heads, const uint8_t* k_fp8,
                          const float* k_scale, int64_t n_tokens, const float* weights,
                          const int32_t* row_start, const int32_t* row_end, float* logits,
                          int64_t logits_stride, int16_t* mask, hcu_stream_t stream);

/* Fused prefill indexer (new; no counterpart in the reference, whose prefill
 * indexer is the closed lightop _mqa_logits followed by the materialised
 * top-k): the result of hcu_mqa_logits_ragged (row_start = 0) followed by
 * hcu_sparse_mask_topk_transform (lengths = row_end), without writing the
 * logits.  A sampled pass estimates each row's top-2048 threshold, the full
 * pass appends the tokens at or above it to per-row lists, and a select writes
 * their top-2048 in the canonical order; rows whose list cannot prove
 * exactness raise a device flag and are recomputed by the materialising pair,
 * predicated on that flag (no host synchronisation).
 *   q       fp8 [rows, heads, 128]; weights fp32 [rows, heads]
 *   k_fp8   fp8 [n_tokens, 128]; k_scale fp32 [n_tokens]; n_tokens <= 131072
 *   row_end int32 [rows]: row r sees tokens [0, row_end[r])
 *   page_table int32 [rows, >= n_tokens] row stride pt_stride (0: one row for all)
 *   dst     int32 [rows, 2048]
 *   workspace >= hcu_mqa_topk_ragged_workspace_bytes(rows, n_tokens), 16-byte aligned
 *   fallback_flag (nullable) int32 [1]: 1 when the exact path ran. */
int64_t hcu_mqa_topk_ragged_workspace_bytes(int64_t rows, int64_t n_tokens);
int hcu_mqa_topk_ragged(const uint8_t* q, int64_t rows, int64_t heads, const uint8_t* k_fp8,
                        const float* k_scale, int64_t n_tokens, const float* weights,
                        const int32_t* row_end, const int32_t* page_table, int64_t pt_stride,
                        int32_t* dst, void* workspace, int64_t workspace_bytes, int32_t* fallback_flag,
                        hcu_stream_t stream);

/* ------------------------------------------------------------------------
 * Stage 3: exact top-2048 + page-table transform
 * ------------------------------------------------------------------------ */

/* Bytes of workspace the split variants need for [rows, width] scores. */
int64_t hcu_topk_workspace_bytes(int64_t rows, int64_t width, int64_t max_splits);

/* Exact top-k (topk must be 2048) of the masked scores of every row, written
 * through the page table.  Replaces _C.sparse_mask_topk_transform
 * (hcu_ops/csrc/sparse_mask_topk.cu:896-908, bind.cpp:3-6,47-48).
 *   score   fp32 [rows, width] row stride score_stride (elements)
 *   mask    int16 [rows, ceil(width/16)] row stride mask_stride
 *   lengths int32 [rows]; len = min(lengths[r], width)
 *   page_table int32 [rows, >= width] row stride pt_stride
 *   dst     int32 [rows, 2048]
 * Tokens whose mask bit is clear count as +0.  Ties break toward the lower
 * token index.  Output: tokens above the threshold key in ascending token
 * order, then the threshold ties in ascending order; len <= 2048 gives
 * pt[i] for i < len and -1 after. */
int hcu_sparse_mask_topk_transform(const float* score, int64_t rows, int64_t width, int64_t score_stride,
                                   const int16_t* mask, int64_t mask_stride, const int32_t* lengths,
                                   const int32_t* page_table, int64_t pt_stride, int64_t topk,
                                   int32_t* dst, hcu_stream_t stream);

/* Same result; a row is spread over up to max_splits CTAs when rows are few
 * (replaces _C.sparse_mask_topk_transform_split, sparse_mask_topk.cu:910-981):
 * min(ceil(width / 8192), SMs / rows, max_splits, 8) CTAs per row, launched as
 * one thread-block cluster per row, each taking at least 8192 of the row's
 * visible tokens.  The workspace is not used (hcu_topk_workspace_bytes = 0). */
int hcu_sparse_mask_topk_transform_split(const float* score, int64_t rows, int64_t width,
                                         int64_t score_stride, const int16_t* mask, int64_t mask_stride,
                                         const int32_t* lengths, const int32_t* page_table,
                                         int64_t pt_stride, int64_t topk, int64_t max_splits,
                                         void* workspace, int64_t workspace_bytes, int32_t* dst,
                                         hcu_stream_t stream);

/* List strategy for many rows (new; serves the same call as
 * hcu_sparse_mask_topk_transform, sparse_mask_topk.cu:896-908, with a caller
 * workspace like the split variants').  One warp per row derives a bound from
 * 2048 samples of the row; one warp per row streams the row into a list of the
 * tokens at or above it; the top 2048 of each list are written in the canonical
 * order; a row whose list cannot prove exactness is rewritten by the plain
 * kernel, launched last and predicated per row.  Same arguments and result as
 * hcu_sparse_mask_topk_transform; width <= 131072; workspace 256-byte aligned,
 * at least hcu_sparse_mask_topk_transform_lists_workspace_bytes(rows, width)
 * (about 64 KiB per row), no initial contents needed. */
int64_t hcu_sparse_mask_topk_transform_lists_workspace_bytes(int64_t rows, int64_t width);
int hcu_sparse_mask_topk_transform_lists(const float* score, int64_t rows, int64_t width,
                                         int64_t score_stride, const int16_t* mask, int64_t mask_stride,
                                         const int32_t* lengths, const int32_t* page_table,
                                         int64_t pt_stride, int64_t topk, void* workspace,
                                         int64_t workspace_bytes, int32_t* dst, hcu_stream_t stream);

/* Split variant whose pass 1 was built by hcu_mqa_logits_hist(hist_lens=lengths)
 * into zws (replaces _C.sparse_mask_topk_transform_split_pre, sparse_mask_topk.cu:986-1051). */
int hcu_sparse_mask_topk_transform_split_pre(const float* score, int64_t rows, int64_t width,
                                             int64_t score_stride, const int16_t* mask,
                                             int64_t mask_stride, const int32_t* lengths,
                                             const int32_t* page_table, int64_t pt_stride,
                                             int64_t topk, int64_t max_splits, int32_t* zws,
                                             void* workspace, int64_t workspace_bytes, int32_t* dst,
                                             hcu_stream_t stream);

/* Allocation-free top-k (no counterpart in the reference).  For callers that
 * cannot allocate device memory -- code inside an engine that owns the device's
 * memory pool, or a plug-in run where a cudaMalloc would synchronise the device
 * or exceed its budget.  Same arguments and result as
 * hcu_sparse_mask_topk_transform; internally it builds the pass-1 histogram of
 * the split_pre path in one fixed device array of this library (8 MiB, held by
 * every GPU that loads the library until the process exits) and allocates
 * nothing.  Limits and rules:
 *   - rows <= hcu_topk_noalloc_max_rows() (256); larger batches return
 *     HCU_ERR_ARG with a message in hcu_last_error_string();
 *   - the array is shared by every call on a device: calls that may overlap on
 *     the GPU (different streams without ordering) race and must not be issued;
 *     each call rewrites the part it reads, so back-to-back calls are fine;
 *   - the first call on a device looks up the array's device address (a CUDA
 *     runtime call); make that first call before any stream capture. */
int hcu_sparse_mask_topk_transform_noalloc(const float* score, int64_t rows, int64_t width,
                                           int64_t score_stride, const int16_t* mask, int64_t mask_stride,
                                           const int32_t* lengths, const int32_t* page_table, int64_t pt_stride,
                                           int64_t topk, int32_t* dst, hcu_stream_t stream);

/* Largest row count hcu_sparse_mask_topk_transform_noalloc accepts. */
int64_t hcu_topk_noalloc_max_rows(void);

/* Top-k that also returns the selected keys (the monotone uint32 image of the
 * fp32 score; +0 = 0x80000000 for unset mask bits; 0 for -1 pads).  Used by the
 * context-parallel path; same selection and order as hcu_sparse_mask_topk_transform. */
int hcu_topk_keys(const float* score, int64_t rows, int64_t width, int64_t score_stride,
                  const int16_t* mask, int64_t mask_stride, const int32_t* lengths,
                  const int32_t* page_table, int64_t pt_stride, int32_t* dst, uint32_t* dst_keys,
                  hcu_stream_t stream);

/* ------------------------------------------------------------------------
 * Context-parallel merge (new): P per-range (key, global index) lists per row
 * -> the global top-2048, in the single-GPU canonical order.
 *   keys    uint32 [P, rows, 2048]; gidx int32 [P, rows, 2048] (-1 pads); part p
 *           lists its candidates in ascending global index and parts cover
 *           ascending contiguous ranges
 *   lengths int32 [rows] total visible tokens of each row (<= 2048: keep all in
 *           index order; else the canonical top-k order)
 *   dst     int32 [rows, 2048] global token indices (-1 pads)
 * ------------------------------------------------------------------------ */
int hcu_cp_topk_merge(const uint32_t* keys, const int32_t* gidx, int64_t n_parts, int64_t rows,
                      const int32_t* lengths, int32_t* dst, hcu_stream_t stream);

/* Context-parallel bounded exchange (no counterpart in the reference, whose CP8
 * splits the queries instead; see hcu_ops/cp.py).  Three steps per rank:
 *
 * hcu_cp_local_bound: per row an order-preserving int32 (key ^ 0x80000000) of a
 * sampled estimate of the row's global top-2048 threshold on this rank's range
 * (lengths = visible tokens in the range, totals = visible tokens of the whole
 * row); rows with totals <= 2048 and empty ranges give INT32_MAX.  The caller
 * takes the minimum over ranks (an all-reduce MIN) as the row's bound. */
int hcu_cp_local_bound(const float* score, int64_t rows, int64_t width, int64_t score_stride,
                       const int16_t* mask, int64_t mask_stride, const int32_t* lengths, const int32_t* totals,
                       int32_t* bounds, hcu_stream_t stream);

/* hcu_cp_filter: every token of the row's range with key >= bound, in token
 * order, as (key, page_table entry) into cap (<= 2048) slots; key 0 / entry -1
 * pads.  Row r's list starts at (r / rows_per_block) * block_stride +
 * (r % rows_per_block) * cap of keys and of gidx, so the lists land directly in
 * a row-sharded exchange buffer.  counts (optional) = tokens at or above the
 * bound; *flag |= 1 when a row has more than cap of them. */
int hcu_cp_filter(const float* score, int64_t rows, int64_t width, int64_t score_stride, const int16_t* mask,
                  int64_t mask_stride, const int32_t* lengths, const int32_t* page_table, int64_t pt_stride,
                  const int32_t* bounds, int64_t cap, uint32_t* keys, int32_t* gidx, int64_t rows_per_block,
                  int64_t block_stride, int32_t* counts, int32_t* flag, hcu_stream_t stream);

/* hcu_cp_topk_merge with lists of list_len (a power of two in [256, 2048],
 * n_parts * list_len >= 2048) entries, part p's lists at p * part_stride.
 * flag (optional): *flag |= 1 for a row longer than 2048 tokens whose lists hold
 * fewer than 2048 entries (a bound that missed; without flag such input sets
 * HCU_STATUS_BAD_INPUT).  short_identity: rows of at most 2048 visible tokens
 * are written as 0, 1, .., len - 1 (identity page table) without reading lists. */
int hcu_cp_topk_merge_lists(const uint32_t* keys, const int32_t* gidx, int64_t n_parts, int64_t list_len,
                            int64_t part_stride, int64_t rows, const int32_t* lengths, int32_t* flag,
                            int32_t short_identity, int32_t* dst, hcu_stream_t stream);

/* ------------------------------------------------------------------------
 * Context-parallel exchange over peer memory (no counterpart in the reference).
 *
 * The same bounded exchange as above, with each exchange fused into the kernel
 * that produces its data: every rank's buffers below are mapped into every
 * other rank's address space (CUDA IPC / symmetric memory over NVLink), the
 * kernels store straight into the destination rank's buffer and publish their
 * completion with a per-step flag (system-scope release store); the consumer
 * kernels wait for the flags of all ranks (bounded waits, acquire loads).  A
 * step is, per rank, in stream order:
 *   hcu_cp_peer_bound   bounds of this range -> slot `rank` of every rank's bounds
 *   hcu_cp_peer_filter  waits for all bounds, takes their minimum per row, stores
 *                       each row's list into slot `rank` of the row owner's lists
 *   hcu_cp_peer_merge   waits for all lists of this rank's rows, merges them and
 *                       stores each result row into every rank's out
 *   hcu_cp_peer_finish  waits for every rank's rows; ws[HCU_CP_WS_FLAG] = 1 when
 *                       any rank flagged a row (the bounded exchange was not exact)
 * and then, predicated on that flag on the device (identical on every rank, so
 * all ranks take the same branch and no host read is needed), the exact redo:
 *   hcu_topk_keys_if          local top-2048 with keys of every row
 *   hcu_cp_peer_scatter_exact lists -> slot `rank` of the row owner's lists_exact
 *   hcu_cp_peer_merge         (exact = 1) merge of the 2048-entry lists
 *   hcu_cp_peer_finish        (exact = 1) ws[HCU_CP_WS_RERUNS] += 1
 * Rank d owns rows [d * rps, (d + 1) * rps).  Every buffer is written by one rank
 * per slot, so no two ranks write the same word.  `epoch` starts at 1 and grows
 * by 1 per step; flags hold (epoch << 1 | flag bit).  The result in out is valid
 * until the next step's merge of any rank.
 * ------------------------------------------------------------------------ */
#define HCU_CP_MAX_PARTS 16
enum {
  HCU_CP_WS_FLAG = 8,    /* ws word: this step's bounded exchange was flagged (the exact redo ran) */
  HCU_CP_WS_RERUNS = 9,  /* ws word: number of exact redos so far */
  HCU_CP_WS_WORDS = 16,  /* int32 words of ws (zeroed before the first step) */
  HCU_CP_SIG_WORDS = 5   /* signal words per source rank (x parts) */
};
typedef struct {
  int32_t parts;         /* P <= HCU_CP_MAX_PARTS */
  int32_t rank;          /* this rank */
  int32_t rows;          /* query rows R (the same on every rank) */
  int32_t rows_per_rank; /* rps = ceil(R / P) */
  int32_t list_len;      /* C: slots per (rank, row) list of the bounded exchange (power of two, 256..2048) */
  uint32_t epoch;        /* step number, from 1 */
  int32_t* ws;           /* this rank's local workspace, HCU_CP_WS_WORDS int32 */
  int32_t* bounds[HCU_CP_MAX_PARTS];      /* rank p's int32 [P, R] */
  int32_t* lists[HCU_CP_MAX_PARTS];       /* rank p's int32 [P, 2, rps, C]: keys then entries */
  int32_t* lists_exact[HCU_CP_MAX_PARTS]; /* rank p's int32 [P, 2, rps, 2048] */
  int32_t* out[HCU_CP_MAX_PARTS];         /* rank p's int32 [P * rps, 2048] result */
  uint32_t* sig[HCU_CP_MAX_PARTS];        /* rank p's uint32 [HCU_CP_SIG_WORDS, P] flags */
} hcu_cp_peers_t;

/* lengths: this range's visible tokens per row; totals: each row's visible
 * tokens over all ranges.  Score / mask as hcu_cp_local_bound. */
int hcu_cp_peer_bound(const float* score, int64_t width, int64_t score_stride, const int16_t* mask,
                      int64_t mask_stride, const int32_t* lengths, const int32_t* totals,
                      const hcu_cp_peers_t* peers, hcu_stream_t stream);

/* page_table: [R, >= width] global token index of each local token (as hcu_cp_filter). */
int hcu_cp_peer_filter(const float* score, int64_t width, int64_t score_stride, const int16_t* mask,
                       int64_t mask_stride, const int32_t* lengths, const int32_t* page_table,
                       int64_t pt_stride, const hcu_cp_peers_t* peers, hcu_stream_t stream);

/* totals: visible tokens of this rank's rows (rps entries; rows past R: 0).
 * exact = 0: the bounded lists; exact = 1: the 2048-entry lists of the redo
 * (does nothing unless ws[HCU_CP_WS_FLAG] is set). */
int hcu_cp_peer_merge(const int32_t* totals, int32_t exact, const hcu_cp_peers_t* peers, hcu_stream_t stream);

/* keys / entries: this rank's hcu_topk_keys output for all R rows ([R, 2048]).
 * Does nothing unless ws[HCU_CP_WS_FLAG] is set. */
int hcu_cp_peer_scatter_exact(const uint32_t* keys, const int32_t* entries, const hcu_cp_peers_t* peers,
                              hcu_stream_t stream);

int hcu_cp_peer_finish(int32_t exact, const hcu_cp_peers_t* peers, hcu_stream_t stream);

/* hcu_topk_keys that does nothing unless *run_if != 0 (a device word). */
int hcu_topk_keys_if(const float* score, int64_t rows, int64_t width, int64_t score_stride,
                     const int16_t* mask, int64_t mask_stride, const int32_t* lengths,
                     const int32_t* page_table, int64_t pt_stride, int32_t* dst, uint32_t* dst_keys,
                     const int32_t* run_if, hcu_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* HCU_INDEXER_H_ */
