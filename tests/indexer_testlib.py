"""Shared test helpers: score generators, validity criteria and tolerances.

``make_scores`` restates the reference's ten top-k score distributions
(``hcu_ops/tests/topk_lib.py:8-51``) on a seeded CPU generator; the reference's
own outputs of that generator are stored in ``tests/golden/topk_make_cases.npz``.
``same_values`` restates the reference's validity criterion (``topk_lib.py:70-89``).
"""
from __future__ import annotations

import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DISTS = ["pos", "sparse30", "sparse2", "relu_sum", "mixed", "ties", "zeros", "neg", "narrow", "const"]

# Logits tolerance of the build's contract: |dev - ref| <= RTOL * max(|ref|, floor), where
# floor = 1e-2 * sum_h |w_h| relu(acc_h) |k_scale| guards rows whose head sum cancels.
LOGITS_RTOL = 1e-2


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def make_scores(B, L, dist, W=None, ragged=False, seed=0):
    """Scores [B, W] (NaN where the mask bit is clear), int16 mask, lengths, page table."""
    W = W or L
    g = torch.Generator().manual_seed(seed)

    def rand(*s):
        return torch.rand(*s, generator=g)

    if dist == "pos":
        x = rand(B, W) * 10
    elif dist == "sparse30":
        x = rand(B, W) * 10
        x[rand(B, W) > 0.3] = 0
    elif dist == "sparse2":
        x = rand(B, W) * 10
        x[rand(B, W) > 1500.0 / W] = 0
    elif dist == "relu_sum":
        n = torch.randn(B, W, 8, generator=g)
        x = (torch.relu(n) * (rand(8) - 0.3)).sum(-1)
    elif dist == "mixed":
        x = torch.randn(B, W, generator=g)
    elif dist == "ties":
        x = torch.randint(0, 50, (B, W), generator=g).float() / 4
    elif dist == "zeros":
        x = torch.zeros(B, W)
    elif dist == "neg":
        x = -rand(B, W)
        x[rand(B, W) > 0.5] = 0
    elif dist == "narrow":
        x = 1.0 + rand(B, W) * 1e-3
    elif dist == "const":
        x = torch.full((B, W), 0.5)
    else:
        raise ValueError(dist)
    x = x.float().contiguous()
    nz = (x != 0)
    pad = (-W) % 16
    if pad:
        nz = torch.cat([nz, torch.zeros(B, pad, dtype=torch.bool)], 1)
    w16 = torch.tensor([1 << i for i in range(16)], dtype=torch.int32)
    bits = (nz.view(B, -1, 16).to(torch.int32) * w16).sum(-1, dtype=torch.int32)
    mask = torch.where(bits > 32767, bits - 65536, bits).to(torch.int16).contiguous()
    x = torch.where(x == 0, torch.full_like(x, float("nan")), x)
    if ragged:
        lengths = (L - torch.arange(B) * 37 - 3).clamp(min=1).to(torch.int32)
    else:
        lengths = torch.full((B,), L, dtype=torch.int32)
    pt = (torch.arange(W, dtype=torch.int32).unsqueeze(0).repeat(B, 1)
          + 7 + 1000000 * torch.arange(B, dtype=torch.int32).unsqueeze(1)).contiguous()
    return x, mask, lengths, pt


def same_values(x, lengths, ref, out, pt):
    """Both outputs are valid top-k: equal sorted value multisets, unique indices below the length."""
    xv = np.nan_to_num(np.asarray(x), nan=0.0)
    B = xv.shape[0]
    off = np.asarray(pt)[:, :1].astype(np.int64)

    def vals(o):
        o = np.asarray(o).astype(np.int64)
        idx = o - off
        valid = o >= 0
        v = np.take_along_axis(xv, np.clip(idx, 0, xv.shape[1] - 1), 1)
        return np.sort(np.where(valid, v, -np.inf), -1), idx, valid

    vr, _, _ = vals(ref)
    vo, io, valid = vals(out)
    if not np.array_equal(vr, vo):
        return False
    for b in range(B):
        sel = io[b][valid[b]]
        if np.unique(sel).size != sel.size or (sel >= int(lengths[b])).any():
            return False
    return True


def compare_logits(dev_logits, dev_mask, ref_logits, ref_mask, floor, widths=None, rtol=LOGITS_RTOL):
    """Compare device logits/mask with the oracle under the build's tolerance.

    Returns a dict of diagnostics; ``ok`` requires (a) identical mask bits except
    where the oracle value is itself within tolerance of zero, and (b) at every
    token set in both masks ``|dev - ref| <= rtol * max(|ref|, floor)``.
    """
    from oracle.indexer import mask_bits

    W = ref_logits.shape[1]
    md = mask_bits(np.asarray(dev_mask), W)
    mr = mask_bits(np.asarray(ref_mask), W)
    both = md & mr
    dl = np.asarray(dev_logits)[:, :W]
    rl = np.asarray(ref_logits)
    fl = np.asarray(floor)
    scale = np.maximum(np.abs(np.nan_to_num(rl)), fl)
    err = np.where(both, np.abs(dl - rl), 0.0)
    bad_val = both & ~(err <= rtol * scale)
    diff = md ^ mr
    # a mask difference is only tolerable where the value is indistinguishable from 0
    dv = np.where(md, np.abs(np.nan_to_num(dl)), np.abs(np.nan_to_num(rl)))
    bad_mask = diff & ~(dv <= rtol * np.maximum(fl, 1e-30))
    rel = np.where(both, err / np.maximum(scale, 1e-30), 0.0)
    return dict(ok=not bad_val.any() and not bad_mask.any(), n_bad_val=int(bad_val.sum()),
                n_bad_mask=int(bad_mask.sum()), n_mask_diff=int(diff.sum()), max_rel=float(rel.max(initial=0.0)),
                n_set=int(mr.sum()))


def overlap(a, b):
    """Mean per-row fraction of shared valid entries between two [rows, k] index arrays."""
    fr = []
    for x, y in zip(np.asarray(a), np.asarray(b)):
        sx = set(x[x >= 0].tolist())
        sy = set(y[y >= 0].tolist())
        fr.append(len(sx & sy) / max(len(sx), 1))
    return float(np.mean(fr)) if fr else 1.0


def e2e_vs_oracle(got, ref_logits, ref_mask, floor, lengths, pt, rows=None, rtol=LOGITS_RTOL):
    """End-to-end selection check against the oracle's own logits.

    ``got``: device top-k page-table entries ``[n, 2048]`` for oracle rows ``rows`` (default all);
    ``ref_logits``/``ref_mask``/``floor``: the oracle's logits of those rows.  Returns (overlap,
    n_bad): the mean per-row fraction of the oracle's selection the device also selected, and the
    number of disagreeing tokens that are NOT near-ties -- a token may fall on either side only
    when its oracle value is within the two values' combined tolerance of the oracle's threshold
    (the 2048th largest value of the row)."""
    from oracle.indexer import TOPK, mask_bits, row_keys, select_topk

    got = np.asarray(got)
    rl = np.asarray(ref_logits)
    W = rl.shape[1]
    mb = mask_bits(np.asarray(ref_mask), W)
    fl = np.asarray(floor)
    lens = np.minimum(np.asarray(lengths, dtype=np.int64), W)
    fr, bad = [], 0
    for i in range(got.shape[0]):
        L = int(max(lens[i], 0))
        keys = row_keys(rl[i], mb[i], L)
        sel = select_topk(keys)
        ptr = np.asarray(pt[i][:L]).astype(np.int64)
        ref_set = set(ptr[sel].tolist())
        g = got[i][got[i] >= 0]
        dev_set = set(g.tolist())
        fr.append(len(ref_set & dev_set) / max(len(ref_set), 1))
        if L <= TOPK or ref_set == dev_set:
            continue
        inv = {int(e): t for t, e in enumerate(ptr.tolist())}
        val = np.where(mb[i, :L], np.nan_to_num(rl[i, :L]), 0.0)
        t_thr = int(sel[-1]) if sel.shape[0] == TOPK else int(sel[np.argmin(keys[sel])])
        thr = val[t_thr]
        tol_thr = rtol * max(abs(thr), fl[i, t_thr])
        for e in ref_set ^ dev_set:
            t = inv.get(int(e))
            if t is None:
                bad += 1
                continue
            if abs(val[t] - thr) > rtol * max(abs(val[t]), fl[i, t]) + tol_thr:
                bad += 1
    return float(np.mean(fr)) if fr else 1.0, bad
