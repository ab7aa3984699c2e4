"""GPU parity of the ragged (prefill) logits kernel and of prefill top-k on its output.

Same tolerance contract as the paged kernel (``indexer_testlib.compare_logits``); top-k on
the device's own logits is bit-exact against the oracle."""
import numpy as np
import pytest
import torch

from indexer_testlib import compare_logits, overlap
from oracle import indexer as O

pytestmark = pytest.mark.gpu


def _ragged(rows, prefix, heads, seed, n_tokens=None):
    from hcu_ops.workloads import make_ragged

    return make_ragged(rows, prefix, heads=heads, seed=seed, n_tokens=n_tokens)


def _oracle(w, rows=None):
    R = w["q"].shape[0]
    return O.mqa_logits_ragged(w["q"].view(torch.uint8).numpy().reshape(R, w["heads"], 128),
                               w["k_fp8"].view(torch.uint8).numpy(), w["k_scale"].numpy(), w["weights"].numpy(),
                               w["row_start"].numpy(), w["row_end"].numpy(), want_floor=True, rows=rows)


def _run(hcu, w, dev):
    d = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in w.items()}
    lg, mk = hcu.mqa_logits_ragged(d["q"], d["k_fp8"], d["k_scale"], d["weights"], d["row_start"], d["row_end"])
    return lg, mk, d


CASES = [
    # rows, prefix, heads, n_tokens override
    (1, 0, 64, None),        # one row, one token
    (5, 100, 64, None),      # rows fewer than a row block
    (16, 1000, 64, None),    # exactly one super-block
    (37, 3000, 64, None),    # ragged last super-block
    (40, 2000, 32, None),    # 32 heads: 8 rows per row block
    (64, 8192, 64, None),
    (20, 500, 64, 3000),     # K longer than every row's range (trailing tokens never visible)
]


@pytest.mark.parametrize("case", CASES, ids=[f"r{c[0]}p{c[1]}h{c[2]}" for c in CASES])
def test_ragged_logits_vs_oracle(hcu, dev, case):
    rows, prefix, heads, n_tok = case
    w = _ragged(rows, prefix, heads, seed=rows + prefix, n_tokens=n_tok)
    lg, mk, _ = _run(hcu, w, dev)
    rl, rm, fl = _oracle(w)
    assert lg.shape == rl.shape and mk.shape == rm.shape
    res = compare_logits(lg.cpu().numpy(), mk.cpu().numpy(), rl, rm, fl)
    assert res["ok"], res


def test_ragged_nan_inputs_follow_fmaxf(hcu, dev):
    """NaN fp8 bytes (e4m3fn 0x7F / 0xFF) in K and q: the reference's ReLU is fmaxf, so a NaN dot
    product contributes 0 and every stored logit is finite (the saturating-FMA ReLU flushes NaN
    to +0)."""
    w = _ragged(16, 1000, 64, seed=9)
    kb = w["k_fp8"].view(torch.uint8)
    kb[5, :] = 0x7F          # a whole NaN token (positive NaN dot products)
    kb[700, 3] = 0xFF        # one negative-NaN byte
    kb[1010, 127] = 0x7F
    qb = w["q"].view(torch.uint8).view(w["q"].shape[0], w["heads"], 128)
    qb[2, 7, 0] = 0x7F       # one head of one row
    lg, mk, _ = _run(hcu, w, dev)
    rl, rm, fl = _oracle(w)
    assert np.isfinite(np.where(O.mask_bits(rm, rl.shape[1]), rl, 0.0)).all()
    res = compare_logits(lg.cpu().numpy(), mk.cpu().numpy(), rl, rm, fl)
    assert res["ok"], res
    got = lg.cpu().numpy()
    assert np.isfinite(got[O.mask_bits(mk.cpu().numpy(), got.shape[1])]).all()


def test_ragged_arbitrary_ranges(hcu, dev):
    """Non-causal windows: empty ranges, ranges starting mid-tile, ranges past the end."""
    w = _ragged(24, 1500, 64, seed=4)
    g = torch.Generator().manual_seed(4)
    start = torch.randint(0, 1400, (24,), generator=g, dtype=torch.int32)
    length = torch.randint(0, 600, (24,), generator=g, dtype=torch.int32)
    start[3], length[3] = 100, 0            # empty
    start[5], length[5] = 1500, 5000        # runs past n_tokens
    start[7], length[7] = -50, 100          # starts before 0
    w["row_start"], w["row_end"] = start, (start + length).to(torch.int32)
    lg, mk, _ = _run(hcu, w, dev)
    rl, rm, fl = _oracle(w)
    res = compare_logits(lg.cpu().numpy(), mk.cpu().numpy(), rl, rm, fl)
    assert res["ok"], res
    assert (mk[3] == 0).all()


def test_prefill_topk_on_device_logits(hcu, dev):
    """Prefill pipeline: ragged logits -> top-2048 (token indices through an identity table)."""
    rows, prefix = 48, 6000
    w = _ragged(rows, prefix, 64, seed=9)
    lg, mk, d = _run(hcu, w, dev)
    N = lg.shape[1]
    lens = d["row_end"]
    ident = torch.arange(N, dtype=torch.int32, device=dev).repeat(rows, 1)
    cu = torch.arange(rows + 1, dtype=torch.int32, device=dev)
    score = lg.contiguous()
    out = hcu._C.sparse_mask_topk_transform(score, mk.contiguous(), lens, ident, cu, 2048)
    ref = O.topk_transform(score.cpu().numpy(), mk.cpu().numpy(), lens.cpu().numpy(), ident.cpu().numpy())
    assert np.array_equal(out.cpu().numpy(), ref)
    rl, rm, _ = _oracle(w)
    ref_e2e = O.topk_transform(rl, rm, lens.cpu().numpy(), ident.cpu().numpy())
    assert overlap(out.cpu().numpy(), ref_e2e) >= 0.999


def test_ragged_matches_paged_kernel(hcu, dev):
    """The same rows through both kernels (identity block table) agree to fp32 rounding."""
    from hcu_ops.workloads import pack_index_k_pages

    rows, prefix = 8, 700
    w = _ragged(rows, prefix, 64, seed=2, n_tokens=768)
    lg, mk, d = _run(hcu, w, dev)
    kv = pack_index_k_pages(d["k_fp8"], d["k_scale"])
    bt = torch.arange(12, dtype=torch.int32, device=dev).repeat(rows, 1)
    plg, pmk, _ = hcu._C.mqa_logits_hist(d["q"].view(rows, 1, 64, 128), kv, d["weights"], d["row_end"], bt, 768, 1,
                                         0, 0, None)
    assert torch.equal(pmk, mk)
    m = O.mask_bits(mk.cpu().numpy(), 768)
    a, b = lg.cpu().numpy()[m], plg.cpu().numpy()[m]
    assert np.allclose(a, b, rtol=1e-5, atol=1e-7)
