"""B200 (sm_100a) DSA lightning-indexer ops for sglang's dsa_indexer / dsa_indexer_metadata.

Drop-in for the indexer part of the reference package ``hcu_ops``
(``hcu_ops/hcu_ops/__init__.py:1-105`` of charliedhw/sglang0.5.18-opt): the same
public functions (``sparse_mask_topk_transform``, ``mqa_logits_supported``,
``mqa_logits``), the same ``_C`` op names and layouts, the same environment
switches read once at import, and the same hand-off of the fused pass-1
histogram from ``mqa_logits`` to the next ``sparse_mask_topk_transform``.
Added: the paged K-cache dequant drop-in, the indexer-K dequant, ragged
(prefill) logits, top-k with keys and the context-parallel merge.

All compute runs in ``libhcu_indexer.so`` (hand-written CUDA for sm_100a)
behind ``_C``.  There is no fallback: importing this package fails if the
extension has not been built (``python build.py`` next to this package).
"""
import os

import torch  # noqa: F401  (loads libtorch before the extension)

from . import _C  # noqa: E402  -- ImportError here means the CUDA library is not built

# --------------------------------------------------------------------------- switches
# Call-site switches of the reference's sglang hooks (read by the integration
# layer; kept with the reference's names and defaults).
SGLANG_HCU_MQA_LOGITS = os.environ.get("SGLANG_HCU_MQA_LOGITS", "0") == "1"
SGLANG_HCU_MQA_HIST = os.environ.get("SGLANG_HCU_MQA_HIST", "0") == "1"
SGLANG_HCU_FAST_MASK_TOPK = os.environ.get("SGLANG_HCU_FAST_MASK_TOPK", "1") == "1"
SGLANG_DSA_FAST_DEQUANT_PAGED = os.environ.get("SGLANG_DSA_FAST_DEQUANT_PAGED", "0") == "1"
SGLANG_DSA_FAST_DEQUANT_TOKENS = int(os.environ.get("SGLANG_DSA_FAST_DEQUANT_TOKENS", "8"))
SGLANG_DSA_FAST_DEQUANT_WARPS = int(os.environ.get("SGLANG_DSA_FAST_DEQUANT_WARPS", "4"))

# HCU_TOPK_IMPL: "split" lets a long row be shared by a thread-block cluster of up to HCU_TOPK_SPLITS
# CTAs when the batch leaves SMs idle; "single" keeps every row on one CTA.
_TOPK_IMPL = os.environ.get("HCU_TOPK_IMPL", "split")
_TOPK_SPLITS = int(os.environ.get("HCU_TOPK_SPLITS", "8"))
# HCU_TOPK_LISTS: with at least two rows per SM (prefill chunks, one-GPU context parallelism) and
# widths in (8192, 131072], a warp per row streams the row into a short candidate list above a
# sampled bound and the lists are selected (same result); "0" keeps one CTA per row.
_TOPK_LISTS = os.environ.get("HCU_TOPK_LISTS", "1") == "1"

# Logits tuning knobs of the reference API.  The B200 kernel schedules its
# persistent CTAs from the SM count and the lengths on the device, so
# persistent_ctas / rows_per_cta are accepted as hints only.
_MQA_PCTAS = int(os.environ.get("HCU_MQA_PCTAS", "-1"))
_MQA_PCTAS_G1 = int(os.environ.get("HCU_MQA_PCTAS_G1", str(_MQA_PCTAS)))
_MQA_RPC = int(os.environ.get("HCU_MQA_RPC", "3"))
_MQA_HIST_MAX_ROWS = int(os.environ.get("HCU_MQA_HIST_MAX_ROWS", "8"))
_MQA_HIST_MAX_ROWS_G6 = int(os.environ.get("HCU_MQA_HIST_MAX_ROWS_G6", "0"))
_MQA_HIST = None  # (logits, hist_lens, zws) of the last mqa_logits with a fused histogram
_N_CU = None

SUPPORTED_HEADS = (32, 64)


def _n_sm():
    global _N_CU
    if _N_CU is None:
        _N_CU = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return _N_CU


def _topk_splits(rows, width):
    """Splits sparse_mask_topk_transform_split uses for [rows, width] scores
    (``hcu_ops/hcu_ops/__init__.py:52-57`` of the reference)."""
    return min(max((width + 8191) // 8192, 1), _n_sm() // max(rows, 1), min(_TOPK_SPLITS, 64))


def sparse_mask_topk_transform(score, nonzero_mask, lengths, page_table_size_1, cu_seqlens_q, topk=2048):
    """Exact top-2048 + page-table transform (drop-in for lightop
    fast_topk_transform_sparse_mask_fused; ``__init__.py:15-32`` of the reference).

    Consumes the pass-1 histogram of the preceding ``mqa_logits(..., hist_lens=lengths)``
    when it was built for this very ``score`` and ``lengths``."""
    global _MQA_HIST
    st = _MQA_HIST
    if st is not None:
        _MQA_HIST = None
        if st[0] is score and st[1].data_ptr() == lengths.data_ptr() and st[1].shape == lengths.shape:
            return _C.sparse_mask_topk_transform_split_pre(score, nonzero_mask, lengths, page_table_size_1,
                                                           cu_seqlens_q, topk, _TOPK_SPLITS, st[2])
    if _TOPK_LISTS and 8192 < score.shape[1] <= 131072 and score.shape[0] >= 2 * _n_sm():
        return _C.sparse_mask_topk_transform_lists(score, nonzero_mask, lengths, page_table_size_1, cu_seqlens_q,
                                                   topk)
    if _TOPK_IMPL == "single":
        return _C.sparse_mask_topk_transform(score, nonzero_mask, lengths, page_table_size_1, cu_seqlens_q, topk)
    return _C.sparse_mask_topk_transform_split(score, nonzero_mask, lengths, page_table_size_1, cu_seqlens_q,
                                               topk, _TOPK_SPLITS)


def mqa_logits_supported(q, kv_cache, weights, group_size, context_lens=None, block_table=None,
                         max_context_len=None):
    """Whether mqa_logits takes these operands (else the caller keeps its other path).

    Same contract as ``__init__.py:60-79`` of the reference, widened to 32 or 64
    index heads and any group size that divides the batch."""
    b = q.shape[0] if q.dim() == 4 else 0
    h = q.shape[2] if q.dim() == 4 else 0
    ok = (q.dtype == torch.float8_e4m3fn and q.dim() == 4 and h in SUPPORTED_HEADS
          and tuple(q.shape[1:]) == (1, h, 128) and b > 0 and q.is_contiguous()
          and weights.dtype == torch.float32 and tuple(weights.shape) == (b, h) and weights.is_contiguous()
          and kv_cache.dtype == torch.uint8 and kv_cache.dim() == 4
          and tuple(kv_cache.shape[1:]) == (64, 1, 132) and kv_cache.stride(1) == 132
          and kv_cache.stride(3) == 1 and kv_cache.stride(0) % 16 == 0
          and group_size >= 1 and b % group_size == 0)
    if ok and context_lens is not None:
        ok = (context_lens.dtype == torch.int32 and context_lens.numel() == b and context_lens.is_contiguous())
    if ok and block_table is not None:
        ok = (block_table.dtype == torch.int32 and block_table.dim() == 2 and block_table.shape[0] == b
              and block_table.stride(1) == 1
              and (max_context_len is None or max_context_len == block_table.shape[1] * 64))
    return ok


def mqa_logits(q, kv_cache, weights, context_lens, block_table, max_context_len, group_size,
               hist_lens=None, persistent_ctas=None, rows_per_cta=None):
    """Indexer logits ``(logits [B, max_ctx] f32, mask [B, max_ctx/16] i16)``
    (``__init__.py:82-105`` of the reference).

    Logits hold ``(sum_h w[h] relu(q_h . k)) * k_scale`` where the mask bit is
    set (token < length and the value is not +0) and are unwritten elsewhere.
    hist_lens: lengths of the paired sparse_mask_topk_transform; when that call
    will split rows, its pass-1 histogram is built here and consumed by it."""
    global _MQA_HIST
    rows = q.shape[0]
    if persistent_ctas is None:
        persistent_ctas = _MQA_PCTAS_G1 if group_size == 1 else _MQA_PCTAS
    if rows_per_cta is None:
        rows_per_cta = 1 if group_size == 1 else _MQA_RPC
    if rows_per_cta <= 0 or group_size % rows_per_cta:
        rows_per_cta = 0
    hist_max_rows = _MQA_HIST_MAX_ROWS if group_size == 1 else _MQA_HIST_MAX_ROWS_G6
    use_hist = (hist_lens is not None and _TOPK_IMPL == "split" and rows <= hist_max_rows
                and hist_lens.dtype == torch.int32 and hist_lens.dim() == 1
                and hist_lens.shape[0] == rows and hist_lens.is_contiguous()
                and _topk_splits(rows, max_context_len) > 1)
    logits, mask, zws = _C.mqa_logits_hist(q, kv_cache, weights, context_lens.view(-1), block_table,
                                           max_context_len, group_size, persistent_ctas, rows_per_cta,
                                           hist_lens if use_hist else None)
    _MQA_HIST = (logits, hist_lens, zws) if use_hist else None
    return logits, mask


# --------------------------------------------------------------------------- dequant
def dequantize_k_cache_paged(quant_k_cache, page_table_1_flattened, group_size: int = 128):
    """MLA 656-byte slot paged dequant -> bf16 ``[n, 1, 576]``.

    The arithmetic of ``prefill/patches/patch_fast_dequant.py:45-98`` (fp32
    multiply by the group scale, one round-to-nearest-even to bf16, rope copied
    raw).  Only the 656-byte / group-128 layout exists here; for anything else
    use ``make_dequantize_k_cache_paged`` with sglang's original as fallback."""
    if group_size != 128 or quant_k_cache.shape[-1] != 656:
        raise NotImplementedError("hcu_ops dequant supports the 656-byte slot with group_size=128 only")
    return _C.dequantize_k_cache_paged(quant_k_cache, page_table_1_flattened)


def make_dequantize_k_cache_paged(original):
    """The patched sglang ``dequantize_k_cache_paged``: ours when
    SGLANG_DSA_FAST_DEQUANT_PAGED=1 and the layout is the 656-byte slot, else
    ``original`` (the switch and fallback rule of ``patch_fast_dequant.py:74-84``)."""

    def dequantize_k_cache_paged_hcu(quant_k_cache, page_table_1_flattened, group_size: int = 128):
        if not SGLANG_DSA_FAST_DEQUANT_PAGED or group_size != 128 or quant_k_cache.shape[-1] != 656:
            return original(quant_k_cache, page_table_1_flattened, group_size)
        return _C.dequantize_k_cache_paged(quant_k_cache, page_table_1_flattened)

    return dequantize_k_cache_paged_hcu


def dequant_index_k_paged(kv_cache, token_loc):
    """Indexer-K pages ``[blocks, 64, 1, 132]`` gathered at ``token_loc`` -> bf16 ``[n, 128]``."""
    return _C.dequant_index_k_paged(kv_cache, token_loc)


# --------------------------------------------------------------------------- prefill / CP
def mqa_logits_ragged(q, k_fp8, k_scale, weights, row_start, row_end):
    """Prefill logits: row r over tokens ``[row_start[r], row_end[r])`` of a contiguous fp8 K.

    Returns ``(logits [rows, n_tokens] f32, mask [rows, ceil(n_tokens/16)] i16)``
    with the ``mqa_logits`` contract (logits valid only at set mask bits)."""
    return _C.mqa_logits_ragged(q, k_fp8, k_scale, weights, row_start, row_end)


def mqa_topk_ragged(q, k_fp8, k_scale, weights, row_end, page_table=None, fallback_flag=None):
    """Fused prefill indexer: the top-2048 of ``mqa_logits_ragged(q, k_fp8, k_scale, weights, 0, row_end)``
    through ``page_table`` -- equal to ``sparse_mask_topk_transform`` on those logits with
    ``lengths = row_end`` -- without writing the logits.

    Row r sees tokens ``[0, row_end[r])`` of at most 131072.  ``page_table``: int32 ``[rows, >= tokens]``
    (default: the token index).  ``fallback_flag`` (optional int32 CUDA tensor): set to 1 when some
    row's candidate list could not prove exactness and the materialising path ran instead."""
    if page_table is None:
        n = k_fp8.shape[0]
        page_table = torch.arange(n, dtype=torch.int32, device=q.device).expand(q.shape[0], n)
    return _C.mqa_topk_ragged(q, k_fp8, k_scale, weights, row_end, page_table, fallback_flag)


def quant_store_index_k(k, token_loc, kv_cache):
    """Indexer-K cache writer: quantise each K row (fp32 or bf16 ``[n, 128]``) per token to fp8 e4m3 with an
    fp32 scale ``max(amax, 1e-12) / 448`` and store it into slot ``token_loc[i] = page * 64 + offset`` of
    ``kv_cache`` (uint8 ``[blocks, 64, 1, 132]``, the layout ``mqa_logits`` reads), in place.

    sglang's own store for this cache is not part of the reference's sources; this is the producer of the
    page layout of ``hcu_ops/csrc/mqa_hist.cu:77-91``."""
    return _C.quant_store_index_k(k, token_loc, kv_cache)


def topk_keys(score, nonzero_mask, lengths, page_table):
    """Top-2048 through ``page_table`` plus the selected uint32 keys, in ascending token order."""
    return _C.topk_keys(score, nonzero_mask, lengths, page_table)


def cp_topk_merge(keys, gidx, lengths):
    """Merge per-range (key, global index) lists ``[P, rows, 2048]`` into the global top-2048.

    ``lengths``: total visible tokens per row (selects index order for rows of at most 2048)."""
    return _C.cp_topk_merge(keys, gidx, lengths)


def cp_local_bound(score, nonzero_mask, lengths, totals):
    """Per-row sampled estimate of the row's global top-2048 threshold on this KV range, as an
    order-preserving int32 (key ^ 0x80000000); the context-parallel bound is its minimum over ranks."""
    return _C.cp_local_bound(score, nonzero_mask, lengths, totals)


def cp_filter(score, nonzero_mask, lengths, page_table, bounds, send, flag):
    """Tokens with key >= bound, in token order, into the exchange buffer ``send`` int32
    ``[P, 2, rows per rank, C]`` (keys, then global indices; -1 pads); ``flag[0] |= 1`` when a row
    has more than C of them."""
    _C.cp_filter(score, nonzero_mask, lengths, page_table, bounds, send, flag)


def cp_topk_merge_lists(recv, lengths, flag=None, short_identity=True):
    """Merge the exchanged bounded lists ``recv`` int32 ``[P, 2, rows, C]`` into the global top-2048
    of those rows; ``flag[0] |= 1`` for a row whose lists hold fewer than 2048 entries."""
    return _C.cp_topk_merge_lists(recv, lengths, flag, short_identity)


# --- MLA decode front end (SGLANG_HCU_MLA_KV_FUSED in the reference's sglang patches) --------------
# HCU_NORM_RSQRT_MODE: the rsqrt of the RMS norm (0 and 1: rsqrtf; 2: 1 / sqrtf, IEEE).
_RSQRT_MODE = int(os.environ.get("HCU_NORM_RSQRT_MODE", "0"))


def _rows(x, width):
    """x is [T, width] / [T, 1, width] with a unit last stride."""
    return (x.shape[-1] == width and x.stride(-1) == 1
            and (x.dim() == 2 or (x.dim() == 3 and x.shape[1] == 1)))


def kv_fused_supported(positions, q_pe, q_out, kv_c, kv_weight, k_pe, cos_sin_cache, kv_buffer, loc):
    """Whether rope_qout_kv_store takes these operands (MLA: kv_lora_rank 512, rope 64, bf16,
    656-byte fp8 slots; ``hcu_ops/__init__.py:427-444`` of the reference)."""
    t = positions.numel()
    bf = torch.bfloat16

    def al(x):
        return x.data_ptr() % 16 == 0

    return (q_pe.dtype == bf and q_out.dtype == bf and kv_c.dtype == bf and kv_weight.dtype == bf
            and k_pe.dtype == bf and cos_sin_cache.dtype == bf
            and positions.dtype in (torch.int32, torch.int64) and positions.is_contiguous()
            and q_pe.dim() == 3 and q_pe.shape[0] == t and q_pe.shape[2] == 64 and q_pe.stride(2) == 1
            and q_out.shape == q_pe.shape and q_out.stride(2) == 1
            and cos_sin_cache.dim() == 2 and cos_sin_cache.shape[1] == 64 and cos_sin_cache.is_contiguous()
            and _rows(kv_c, 512) and kv_c.shape[0] == t and kv_c.stride(0) % 8 == 0
            and _rows(k_pe, 64) and k_pe.shape[0] == t
            and kv_weight.is_contiguous() and kv_weight.numel() == 512
            and kv_buffer.dtype == torch.uint8 and kv_buffer.dim() >= 2
            and kv_buffer.numel() // max(kv_buffer.shape[0], 1) >= 656 and kv_buffer.stride(0) % 16 == 0
            and loc.dtype == torch.int64 and loc.is_contiguous() and loc.numel() <= t
            and al(kv_c) and al(kv_weight) and al(kv_buffer))


def rope_qout_kv_store(positions, q_pe, q_out, kv_c, kv_weight, norm_eps, k_pe, cos_sin_cache, is_neox,
                       kv_buffer, loc, store_eps=1e-6):
    """One launch for sglang's DSA decode front end (``hcu_ops/__init__.py:447-455`` of the reference):
    kv_c = rms_norm(kv_c, kv_weight, norm_eps) in place, q_out = rope(q_pe) (q_out may be q_pe),
    k_pe = rope(k_pe) in place, and the fp8 656-byte slots kv_buffer[loc] (512 fp8 in four
    128-element groups, 4 fp32 scales, the rotated k_pe as bf16)."""
    _C.rope_qout_kv_store(positions.reshape(-1), q_pe, q_out, kv_c, kv_weight, float(norm_eps), k_pe,
                          cos_sin_cache, bool(is_neox), kv_buffer, loc, float(store_eps), _RSQRT_MODE)


def read_device_status(clear=True):
    """Sticky device status bits (1: a bounded wait expired, 2: an out-of-range index was skipped)."""
    return _C.read_device_status(clear)


def library_path():
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), "libhcu_indexer.so")
