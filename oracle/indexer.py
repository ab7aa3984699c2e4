"""CPU restatement of the reference's DSA indexer path (test infrastructure only).

Every function names the reference lines it restates. Integer/byte work is
numpy; the fp8 dot products use torch CPU float32 matmul (fp8 x fp8 products
are exact in fp32, so only the fp32 summation order differs from any device).
"""
from __future__ import annotations

import numpy as np
import torch

TOPK = 2048
PAGE = 64
HEAD_DIM = 128
ZERO_KEY = np.uint32(0x80000000)
N_BINS = 4096
ZERO_BIN = 0x800

# ---------------------------------------------------------------------------
# scalar helpers
# ---------------------------------------------------------------------------

_E4M3_LUT = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()


def e4m3_to_f32(b: np.ndarray) -> np.ndarray:
    """fp8 e4m3fn bytes -> exact float32 values (table lookup)."""
    return _E4M3_LUT[np.asarray(b, dtype=np.uint8)]


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """One fp32 -> bf16 round-to-nearest-even, as the device's cvt.rn.bf16.f32.

    Follows the reference dequant's single rounding step
    (``prefill/patches/patch_fast_dequant.py:63-65``: the fp32 product is
    stored through ``.to(bfloat16)``, which rounds to nearest-even on GPUs).
    NaN becomes the canonical bf16 NaN 0x7FFF, which is what the device
    conversion produces; infinities and subnormals round like any value.
    """
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r[nan] = 0x7FFF
    return r


def to_key(x: np.ndarray) -> np.ndarray:
    """Monotone float32 -> uint32 key (``hcu_ops/csrc/sparse_mask_topk.cu:40-43``)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return np.where(b & np.uint32(0x80000000), ~b, b | np.uint32(0x80000000)).astype(np.uint32)


def mask_bits(mask: np.ndarray, width: int) -> np.ndarray:
    """int16 16-token words -> bool [rows, width] (``test_mqa_hist.py:105-106``)."""
    m = np.asarray(mask).astype(np.int64) & 0xFFFF
    bits = (m[..., None] >> np.arange(16)) & 1
    return bits.reshape(m.shape[0], -1)[:, :width].astype(bool)


def pack_mask(bits: np.ndarray) -> np.ndarray:
    """bool [rows, width] -> int16 [rows, ceil(width/16)] (bit j of word i = token 16i+j)."""
    rows, width = bits.shape
    pad = (-width) % 16
    if pad:
        bits = np.concatenate([bits, np.zeros((rows, pad), bool)], 1)
    w = (bits.reshape(rows, -1, 16).astype(np.int64) << np.arange(16)).sum(-1)
    return w.astype(np.uint16).view(np.int16)


# ---------------------------------------------------------------------------
# stage 1: paged K-cache dequant
# ---------------------------------------------------------------------------

def dequant_mla_656(quant_k_cache: np.ndarray, page_table_1: np.ndarray) -> np.ndarray:
    """MLA latent-cache dequant, 656-byte slot -> 576 bf16 (returned as uint16 bits).

    Restates ``prefill/patches/patch_fast_dequant.py:53-71`` (kernel) and
    ``:85-97`` (views): slot = 512 fp8 | 4 fp32 group scales | 64 bf16 rope;
    ``out[t, g*128+j] = bf16_rne(f32(fp8[src, g*128+j]) * scale[src, g])``,
    ``out[t, 512:576] = rope[src]`` copied bit for bit.
    """
    qk = np.ascontiguousarray(quant_k_cache, dtype=np.uint8).reshape(-1, 656)
    src = np.asarray(page_table_1, dtype=np.int64)
    rows = qk[src]
    vals = e4m3_to_f32(rows[:, :512]).reshape(-1, 4, 128)
    scale = np.ascontiguousarray(rows[:, 512:528]).view(np.float32).reshape(-1, 4, 1)
    prod = (vals * scale).astype(np.float32).reshape(-1, 512)
    out = np.empty((src.shape[0], 576), np.uint16)
    out[:, :512] = f32_to_bf16_bits(prod)
    out[:, 512:] = np.ascontiguousarray(rows[:, 528:656]).view(np.uint16)
    return out


def index_k_page_views(kv_pages: np.ndarray):
    """Split indexer-K pages ``[n_pages, 64*132]`` into fp8 ``[n_pages,64,128]`` and f32 ``[n_pages,64]``.

    Page layout from ``hcu_ops/csrc/mqa_hist.cu:77-91``: 64 tokens x 128 fp8
    bytes, then 64 fp32 scales at byte 8192.
    """
    kv = np.ascontiguousarray(kv_pages, dtype=np.uint8).reshape(kv_pages.shape[0], -1)
    fp8 = kv[:, : PAGE * HEAD_DIM].reshape(-1, PAGE, HEAD_DIM)
    sc = np.ascontiguousarray(kv[:, PAGE * HEAD_DIM: PAGE * HEAD_DIM + PAGE * 4]).view(np.float32)
    return fp8, sc


def dequant_index_k(kv_pages: np.ndarray, token_loc: np.ndarray) -> np.ndarray:
    """Indexer-K dequant: ``out[t,:] = bf16_rne(f32(fp8[loc]) * scale[loc])`` (uint16 bits).

    ``token_loc`` is the flattened slot ``page * 64 + offset``; the page
    layout is the one the logits kernel reads (``mqa_hist.cu:77-91``), the
    arithmetic is the reference dequant's (``patch_fast_dequant.py:59-65``).
    """
    fp8, sc = index_k_page_views(kv_pages)
    loc = np.asarray(token_loc, dtype=np.int64)
    page, off = loc // PAGE, loc % PAGE
    vals = e4m3_to_f32(fp8[page, off])
    prod = (vals * sc[page, off][:, None]).astype(np.float32)
    return f32_to_bf16_bits(prod)


def quant_store_index_k(k: np.ndarray, token_loc: np.ndarray, kv_pages: np.ndarray) -> np.ndarray:
    """Indexer-K cache writer (the producer of the page layout ``mqa_hist.cu:77-91``; sglang's
    store is not vendored).  Per token, in float32: ``scale = max(amax, 1e-12) / 448``,
    ``fp8 = e4m3_rne(clamp(x / scale, -448, 448))``; the 128 fp8 bytes go to the slot's row of
    the page, the scale to byte 8192 + 4 * offset.  Returns a written copy of ``kv_pages``
    (uint8 ``[n_pages, page_stride]``); out-of-range slots are skipped.  The arithmetic is the
    per-token amax/448 quantisation the benchmark configs use for K (``hcu_ops/workloads.py``)."""
    x = np.asarray(k, dtype=np.float32).reshape(-1, HEAD_DIM)
    loc = np.asarray(token_loc, dtype=np.int64)
    out = np.array(kv_pages, dtype=np.uint8, copy=True)
    n_pages = out.shape[0]
    amax = np.maximum(np.abs(x).max(axis=1), np.float32(1e-12)).astype(np.float32)
    scale = (amax / np.float32(448.0)).astype(np.float32)
    y = np.clip(x / scale[:, None], np.float32(-448.0), np.float32(448.0)).astype(np.float32)
    q8 = torch.from_numpy(y).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    for t in range(x.shape[0]):
        l = int(loc[t])
        if l < 0 or l >= n_pages * PAGE:
            continue
        pg, off = divmod(l, PAGE)
        out[pg, off * HEAD_DIM:(off + 1) * HEAD_DIM] = q8[t]
        out[pg, PAGE * HEAD_DIM + 4 * off:PAGE * HEAD_DIM + 4 * off + 4] = np.frombuffer(scale[t].tobytes(), np.uint8)
    return out


# ---------------------------------------------------------------------------
# stage 2: MQA index logits + nonzero mask (+ pass-1 histogram)
# ---------------------------------------------------------------------------

def _relu(acc: torch.Tensor) -> torch.Tensor:
    """``fmaxf(acc, 0.0f)`` (``mqa_hist.cu:203``): NaN -> 0."""
    return torch.where(acc > 0, acc, torch.zeros_like(acc))


def _head_sum(acc: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """sum_h relu(acc[h, t]) * w[h] in float32 (``mqa_hist.cu:195-203``).

    The ReLU is ``fmaxf(acc, 0.0f)`` (``:203``): a NaN dot product (from a NaN
    fp8 byte in q or k) contributes 0, like any non-positive one."""
    return (_relu(acc) * w[:, None]).sum(0)


def mqa_logits_paged(q: np.ndarray, kv_pages: np.ndarray, weights: np.ndarray,
                     context_lens: np.ndarray, block_table: np.ndarray,
                     max_context_len: int, group_size: int, want_floor: bool = False):
    """Decode indexer logits over a paged fp8 K cache.

    Restates ``hcu_ops/csrc/mqa_hist.cu``:
      * ``:118-125`` per-row length clamped to ``[0, max_context_len]``;
      * ``:162`` every row of a group of ``group_size`` rows reads the block
        table of the group's first row;
      * ``:195-207`` ``s = (sum_h relu(q_h . k) * w_h) * k_scale``;
      * ``:209-218`` mask bit = ``token < len and bits(s) != 0``, logits
        stored only where the bit is set (elsewhere left NaN here: the
        device leaves that storage unwritten).
    q: uint8 ``[B, H, 128]`` fp8 bytes; weights float32 ``[B, H]``.
    Returns (logits float32 [B, W], mask int16 [B, ceil(W/16)], floor or None);
    ``floor[b, t] = 1e-2 * sum_h |w_h| relu(acc_h) * |k_scale|`` is the
    condition-aware tolerance scale for comparing against a device.
    """
    q = np.asarray(q, dtype=np.uint8)
    B, H, D = q.shape
    assert D == HEAD_DIM
    W = int(max_context_len)
    fp8, sc = index_k_page_views(kv_pages)
    logits = np.full((B, W), np.nan, np.float32)
    keep = np.zeros((B, W), bool)
    floor = np.zeros((B, W), np.float32) if want_floor else None
    qf = torch.from_numpy(e4m3_to_f32(q))
    wf = torch.from_numpy(np.asarray(weights, dtype=np.float32))
    lens = np.clip(np.asarray(context_lens, dtype=np.int64), 0, W)
    bt = np.asarray(block_table, dtype=np.int64)
    for g0 in range(0, B, group_size):
        max_len = int(lens[g0:g0 + group_size].max())
        if max_len == 0:
            continue
        n_pages = (max_len + PAGE - 1) // PAGE
        pages = bt[g0, :n_pages]
        kf = torch.from_numpy(e4m3_to_f32(fp8[pages].reshape(-1, HEAD_DIM))[:max_len])
        ks = torch.from_numpy(sc[pages].reshape(-1)[:max_len].copy())
        for b in range(g0, g0 + group_size):
            L = int(lens[b])
            if L == 0:
                continue
            acc = qf[b] @ kf[:L].T  # [H, L]
            s = _head_sum(acc, wf[b]) * ks[:L]
            sn = s.numpy().astype(np.float32)
            nz = sn.view(np.uint32) != 0
            logits[b, :L][nz] = sn[nz]
            keep[b, :L] = nz
            if want_floor:
                fl = (_relu(acc) * wf[b].abs()[:, None]).sum(0) * ks[:L].abs()
                floor[b, :L] = 1e-2 * fl.numpy()
    return logits, pack_mask(keep), floor


def mqa_logits_ragged(q: np.ndarray, k_fp8: np.ndarray, k_scale: np.ndarray, weights: np.ndarray,
                      row_start: np.ndarray, row_end: np.ndarray, want_floor: bool = False,
                      rows=None):
    """Prefill indexer logits over a contiguous fp8 K with per-row visible range.

    Same per-(row, token) arithmetic and mask contract as ``mqa_logits_paged``
    (``mqa_hist.cu:195-218``) for a query row ``r`` that sees tokens
    ``[row_start[r], row_end[r])`` of ``k_fp8 [N, 128]``. Logits are laid out
    ``[R, N]`` by absolute token index (slots outside the range unset).
    ``rows`` restricts the computation to a subset of rows (CPU baseline).
    """
    q = np.asarray(q, dtype=np.uint8)
    R, H, D = q.shape
    N = k_fp8.shape[0]
    rows = range(R) if rows is None else rows
    logits = np.full((len(rows), N), np.nan, np.float32)
    keep = np.zeros((len(rows), N), bool)
    floor = np.zeros((len(rows), N), np.float32) if want_floor else None
    kf = torch.from_numpy(e4m3_to_f32(k_fp8))
    ks = torch.from_numpy(np.asarray(k_scale, dtype=np.float32))
    wf = torch.from_numpy(np.asarray(weights, dtype=np.float32))
    for i, r in enumerate(rows):
        a, e = int(max(row_start[r], 0)), int(min(row_end[r], N))
        if e <= a:
            continue
        qf = torch.from_numpy(e4m3_to_f32(q[r]))
        acc = qf @ kf[a:e].T
        s = (_head_sum(acc, wf[r]) * ks[a:e]).numpy().astype(np.float32)
        nz = s.view(np.uint32) != 0
        seg = logits[i, a:e]
        seg[nz] = s[nz]
        keep[i, a:e] = nz
        if want_floor:
            fl = (_relu(acc) * wf[r].abs()[:, None]).sum(0) * ks[a:e].abs()
            floor[i, a:e] = 1e-2 * fl.numpy()
    return logits, pack_mask(keep), floor


def pass1_hist(logits: np.ndarray, mask: np.ndarray, hist_lens: np.ndarray, width: int):
    """Fused top-k pass 1: 12-bit key histogram + (positives, zeros) per row.

    Restates ``ref_hist`` (``hcu_ops/tests/test_mqa_hist.py:109-124``) and the
    device contract of ``mqa_hist.cu:219-226,253-271`` + ``:290-303``: rows with
    ``min(hist_len, width) > 2048`` count every set-mask token below that
    length into bin ``key >> 20``, the unset ones (``len - nonzero``) into the
    zero bin 0x800; other rows stay all-zero.
    """
    B = logits.shape[0]
    h = np.minimum(np.asarray(hist_lens, dtype=np.int64), width)
    act = h > TOPK
    mb = mask_bits(mask, width)
    sel = mb & (np.arange(width)[None, :] < h[:, None]) & act[:, None]
    key = to_key(np.where(sel, logits[:, :width], 0.0).astype(np.float32))
    g1 = np.zeros((B, N_BINS), np.int64)
    for b in range(B):
        np.add.at(g1[b], (key[b][sel[b]] >> 20).astype(np.int64), 1)
    nz = sel.sum(1)
    zeros = np.where(act, h - nz, 0)
    g1[:, ZERO_BIN] += zeros
    pos = (sel & (key > ZERO_KEY)).sum(1)
    return g1, np.stack([pos, zeros], 1)


# ---------------------------------------------------------------------------
# stage 3: exact top-2048 + page-table transform
# ---------------------------------------------------------------------------

def row_keys(score_row: np.ndarray, mask_row_bits: np.ndarray, length: int) -> np.ndarray:
    """Keys of tokens ``[0, length)``: unset mask bits are an implicit +0
    (``sparse_mask_topk.cu:83-94``)."""
    v = np.where(mask_row_bits[:length], score_row[:length], 0.0).astype(np.float32)
    k = to_key(v)
    k[~mask_row_bits[:length]] = ZERO_KEY
    return k


def select_topk(keys: np.ndarray, topk: int = TOPK) -> np.ndarray:
    """Canonical selection order for one row of keys (token index = position).

    The 2048 largest keys, ties toward the lower token index; written as the
    tokens strictly above the threshold key in ascending token order, then the
    threshold ties in ascending token order (``sparse_mask_topk.cu:1-7,299-348``).
    Rows with at most ``topk`` tokens select every token in token order
    (``sparse_mask_topk.cu:166-169``).
    """
    n = keys.shape[0]
    if n <= topk:
        return np.arange(n, dtype=np.int64)
    order = np.argsort(~keys, kind="stable")  # key desc, index asc
    thr = keys[order[topk - 1]]
    above = np.nonzero(keys > thr)[0]
    ties = np.nonzero(keys == thr)[0][: topk - above.shape[0]]
    return np.concatenate([above, ties])


def topk_transform(score: np.ndarray, nonzero_mask: np.ndarray, lengths: np.ndarray,
                   page_table_size_1: np.ndarray, topk: int = TOPK,
                   return_keys: bool = False):
    """``sparse_mask_topk_transform``: int32 ``[rows, 2048]`` of page-table entries.

    ``len = min(lengths[r], width)`` (``sparse_mask_topk.cu:161-162``); rows
    with ``len <= 2048`` give ``pt[i]`` for ``i < len`` and -1 after it
    (``:166-169``); other rows give ``pt[idx]`` over ``select_topk``.
    With ``return_keys`` also returns the selected uint32 keys (0 for pads).
    """
    rows, width = score.shape
    mb = mask_bits(nonzero_mask, width)
    out = np.full((rows, topk), -1, np.int32)
    keys_out = np.zeros((rows, topk), np.uint32)
    pt = np.asarray(page_table_size_1)
    lens = np.minimum(np.asarray(lengths, dtype=np.int64), width)
    for r in range(rows):
        L = int(max(lens[r], 0))
        k = row_keys(score[r], mb[r], L)
        idx = select_topk(k, topk)
        out[r, : idx.shape[0]] = pt[r, idx]
        keys_out[r, : idx.shape[0]] = k[idx]
    return (out, keys_out) if return_keys else out


# ---------------------------------------------------------------------------
# context-parallel merge (new in this build; no reference counterpart)
# ---------------------------------------------------------------------------

def cp_merge(keys: np.ndarray, gidx: np.ndarray, lengths: np.ndarray, topk: int = TOPK) -> np.ndarray:
    """Merge per-range top-k lists into the global top-k of one row set.

    ``keys``/``gidx``: ``[P, rows, topk]`` uint32 keys and int32 global token
    indices (-1 pads). The global top-k is a subset of the union of the local
    ones under the total order (key desc, global index asc). The result uses
    the single-range canonical order of ``select_topk`` so it equals the 1-GPU
    output: a row whose total visible length ``lengths[r]`` is at most ``topk``
    -> all candidates in index order; otherwise the above-threshold tokens then
    the ties, each in ascending index order (decided by the visible length, not
    the candidate count: one range may hold all of a longer row's top-k).
    Returns int32 ``[rows, topk]`` global token indices (-1 pads).
    """
    P, rows, K = keys.shape
    out = np.full((rows, topk), -1, np.int32)
    for r in range(rows):
        valid = gidx[:, r, :] >= 0
        k = keys[:, r, :][valid]
        g = gidx[:, r, :][valid].astype(np.int64)
        o = np.argsort(g, kind="stable")
        k, g = k[o], g[o]
        if int(lengths[r]) <= topk:
            sel = np.arange(k.shape[0])
        else:
            order = np.argsort(~k, kind="stable")
            thr = k[order[topk - 1]]
            above = np.nonzero(k > thr)[0]
            sel = np.concatenate([above, np.nonzero(k == thr)[0][: topk - above.shape[0]]])
        out[r, : sel.shape[0]] = g[sel]
    return out


# ---------------------------------------------------------------------------
# context-parallel bounded exchange (this build's CP protocol; the reference's
# CP splits queries instead, so these pin the device ops, not reference code)
# ---------------------------------------------------------------------------

BOUND_SAMPLES = 1024


def _transport(key: np.ndarray) -> np.ndarray:
    """uint32 key -> order-preserving int32 (key ^ 0x80000000)."""
    return (np.asarray(key, dtype=np.uint32) ^ np.uint32(0x80000000)).view(np.int32)


def cp_local_bound(score: np.ndarray, nonzero_mask: np.ndarray, lengths: np.ndarray,
                   totals: np.ndarray) -> np.ndarray:
    """Per-row sampled bound of the row's global top-2048 threshold on one range (device:
    ``cp_bound_kernel``): with n = visible tokens in the range and N = visible tokens of the
    row, m = min(n, 1024) samples (every token when n <= 1024, else 256 groups of 4 consecutive
    tokens starting at min((2g+1) n // 512, n - 4) rounded down to a multiple of 4), t = 2048 m / N,
    r_lo = ceil(t + 3 sqrt(t) + 2); the bound is the r_lo-th largest sample key (1 = largest),
    key 0 when r_lo >= m, the largest key when N <= 2048 or 2048 n < N (n = 0 included).
    Returns int32 [rows] (key ^ 0x80000000)."""
    score = np.asarray(score, dtype=np.float32)
    rows, W = score.shape
    bits = mask_bits(nonzero_mask, W)
    out = np.empty(rows, np.uint32)
    for r in range(rows):
        n = int(np.clip(lengths[r], 0, W))
        N = int(totals[r])
        if N <= TOPK or TOPK * n < N:
            out[r] = 0xFFFFFFFF
            continue
        m = min(n, BOUND_SAMPLES)
        t = np.float32(TOPK) * np.float32(m) / np.float32(N)
        r_lo = int(np.ceil(np.float32(t + np.float32(3.0) * np.sqrt(t) + np.float32(2.0))))
        if r_lo >= m:
            out[r] = 0
            continue
        if n <= BOUND_SAMPLES:
            i = np.arange(n, dtype=np.int64)
        else:
            g = np.arange(BOUND_SAMPLES // 4, dtype=np.int64)
            i0 = np.minimum((2 * g + 1) * n // (2 * (BOUND_SAMPLES // 4)), n - 4) & ~3
            i = (i0[:, None] + np.arange(4)).reshape(-1)
        k = np.where(bits[r, i], to_key(score[r, i]), ZERO_KEY).astype(np.uint32)
        out[r] = np.sort(k)[::-1][r_lo - 1]
    return _transport(out)


def cp_filter(score: np.ndarray, nonzero_mask: np.ndarray, lengths: np.ndarray, page_table: np.ndarray,
              bounds: np.ndarray, cap: int):
    """Tokens of [0, len) with key >= the row's bound, in token order, as (key, page-table entry)
    lists of cap slots (key 0 / entry -1 pads).  A row with more than cap such tokens: with
    cap = 2048, the range's top-2048 among them (canonical selection) in token order; with
    cap < 2048, its top-(cap - 1) in token order and a marker in the last slot (entry -2, key =
    the (cap - 1)-th largest key); past the device's candidate capacity (4096 for widths up to
    32768, else 8192) the flag.  Returns (keys uint32 [rows, cap], gidx int32 [rows, cap],
    counts int32 [rows], flag)."""
    score = np.asarray(score, dtype=np.float32)
    rows, W = score.shape
    bits = mask_bits(nonzero_mask, W)
    lo = (np.asarray(bounds, dtype=np.int32).view(np.uint32) ^ np.uint32(0x80000000)).astype(np.uint32)
    keys = np.zeros((rows, cap), np.uint32)
    gidx = np.full((rows, cap), -1, np.int32)
    counts = np.zeros(rows, np.int32)
    flag = 0
    for r in range(rows):
        n = int(np.clip(lengths[r], 0, W))
        k = np.where(bits[r, :n], to_key(score[r, :n]), ZERO_KEY).astype(np.uint32)
        sel = np.nonzero(k >= lo[r])[0]
        counts[r] = sel.shape[0]
        cand_cap = 4096 if W <= 32768 else 8192
        marker = None
        if cap < sel.shape[0] <= cand_cap:
            kk = cap if cap == TOPK else cap - 1
            order = np.argsort(~k[sel], kind="stable")
            if kk < cap:
                marker = k[sel][order[kk - 1]]
            sel = sel[np.sort(select_topk(k[sel], kk))]
        else:
            flag |= int(sel.shape[0] > cap)
        kept = sel[:cap]
        keys[r, :kept.shape[0]] = k[kept]
        gidx[r, :kept.shape[0]] = np.asarray(page_table)[r, kept]
        if marker is not None:
            keys[r, cap - 1] = marker
            gidx[r, cap - 1] = -2
    return keys, gidx, counts, flag


def cp_merge_lists(keys: np.ndarray, gidx: np.ndarray, lengths: np.ndarray):
    """Merge of bounded lists ``[P, rows, C]``: rows of at most 2048 visible tokens are the
    identity 0..len-1 (device: short_identity); the others are ``cp_merge`` of their lists, and
    a row whose lists hold fewer than 2048 entries, or whose threshold (the 2048th largest key)
    is not above a truncation marker's key (entry -2), raises the flag.  Returns (out, flag)."""
    rows = keys.shape[1]
    out = np.full((rows, TOPK), -1, np.int32)
    flag = 0
    for r in range(rows):
        L = int(lengths[r])
        if L <= TOPK:
            out[r] = np.where(np.arange(TOPK) < L, np.arange(TOPK), -1)
        elif int((gidx[:, r, :] >= 0).sum()) < TOPK:
            flag = 1  # the row's result is not defined; the caller reruns exactly
        else:
            out[r] = cp_merge(keys[:, r:r + 1], gidx[:, r:r + 1], lengths[r:r + 1])[0]
            marks = keys[:, r, :][gidx[:, r, :] == -2]
            if marks.size:
                v = keys[:, r, :][gidx[:, r, :] >= 0]
                thr = np.sort(v)[::-1][TOPK - 1]
                flag |= int(marks.max() >= thr)
    return out, flag
