"""GPU parity of stage 3 (top-2048 + page-table transform): bit-exact, order included,
against the oracle on identical scores -- the reference's distributions, lengths and layouts
(``hcu_ops/tests/test_topk.py:17-48``, ``test_rows.py:9-37`` of the reference)."""
import numpy as np
import pytest
import torch

from indexer_testlib import DISTS, golden, make_scores, same_values
from oracle import indexer as O

pytestmark = pytest.mark.gpu


def _run_all(hcu, x, mask, lens, pt, dev):
    xs, ms, ls, ps = (t.to(dev) for t in (x, mask, lens, pt))
    cu = torch.arange(x.shape[0] + 1, dtype=torch.int32, device=dev)
    C = hcu._C
    return {
        "single": C.sparse_mask_topk_transform(xs, ms, ls, ps, cu, 2048),
        "s8": C.sparse_mask_topk_transform_split(xs, ms, ls, ps, cu, 2048, 8),
        "wrapper": hcu.sparse_mask_topk_transform(xs, ms, ls, ps, cu, 2048),
    }


@pytest.mark.parametrize("dist", DISTS)
@pytest.mark.parametrize("L", [1000, 2048, 2049, 4096, 16384, 65536])
@pytest.mark.parametrize("ragged", [False, True])
def test_topk_exact(hcu, dev, dist, L, ragged):
    if dist in ("zeros", "neg", "ties") and L == 2048:
        pytest.skip("same exclusion as the reference's test grid")
    W = 2 * L + 64 if ragged and L >= 16384 else L + 64  # ragged rows also emulate a padded width
    x, mask, lens, pt = make_scores(6, L, dist, W=W, ragged=ragged, seed=L)
    ref = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy())
    for name, out in _run_all(hcu, x, mask, lens, pt, dev).items():
        got = out.cpu().numpy()
        assert np.array_equal(got, ref), (name, dist, L, ragged)
        assert same_values(x.numpy(), lens.numpy(), ref, got, pt.numpy())


def test_topk_reference_generator_cases(hcu, dev):
    g = golden("topk_make_cases.npz")
    for i in range(int(g["n"])):
        k = f"c{i:02d}"
        x, mask, lens, pt = (torch.from_numpy(g[f"{k}_{n}"]) for n in ("x", "mask", "lengths", "pt"))
        ref = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy())
        for name, out in _run_all(hcu, x, mask, lens, pt, dev).items():
            assert np.array_equal(out.cpu().numpy(), ref), (k, name)


@pytest.mark.parametrize("L", [16384, 65536, 131072])
@pytest.mark.parametrize("dist", ["relu_sum", "narrow"])
def test_topk_production_width(hcu, dev, L, dist):
    """Score width = page-table capacity (1M) under CUDA graphs, ragged rows."""
    x, mask, lens, pt = make_scores(6, L, dist, W=1 << 20, ragged=True, seed=7)
    ref = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy())
    for name, out in _run_all(hcu, x, mask, lens, pt, dev).items():
        assert np.array_equal(out.cpu().numpy(), ref), name


@pytest.mark.parametrize("dist", ["relu_sum", "ties", "sparse2"])
def test_topk_split_rows_mixed_lengths(hcu, dev, dist):
    """One cluster launch (6 rows of width 131136: 8 CTAs per row) whose rows take every path:
    at most 2048 tokens, one CTA's worth (< 2 x 8192 visible tokens: rank 0 alone), and 4, 6
    and 8 CTAs gathering their candidate lists through distributed shared memory."""
    W = 131072 + 64
    x, mask, lens, pt = make_scores(6, 131072, dist, W=W, ragged=False, seed=23)
    lens = torch.tensor([100, 2048, 12000, 32768, 50000, 131072], dtype=torch.int32)
    ref = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy())
    for name, out in _run_all(hcu, x, mask, lens, pt, dev).items():
        assert np.array_equal(out.cpu().numpy(), ref), (name, dist)


@pytest.mark.parametrize("dist", ["relu_sum", "ties", "sparse2"])
def test_topk_many_rows_up_to_96k(hcu, dev, dist):
    """Rows of 60K tokens, more than two per SM: the 512-thread instance (two CTAs per SM)."""
    rows = 2 * torch.cuda.get_device_properties(dev).multi_processor_count + 7
    x, mask, lens, pt = make_scores(rows, 60000, dist, W=60032, ragged=True, seed=41)
    ref = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy())
    for name, out in _run_all(hcu, x, mask, lens, pt, dev).items():
        assert np.array_equal(out.cpu().numpy(), ref), (name, dist)


def test_topk_split_pre_uses_pass1_workspace(hcu, dev):
    x, mask, lens, pt = make_scores(6, 20000, "relu_sum", W=20480, ragged=True, seed=9)
    lens[2] = 1500
    ref = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy())
    g1, cnt = O.pass1_hist(x.numpy(), mask.numpy(), lens.numpy(), 20480)
    zws = np.concatenate([g1.reshape(-1), np.zeros(6 * 4096, np.int64), cnt.reshape(-1)]).astype(np.int32)
    cu = torch.arange(7, dtype=torch.int32, device=dev)
    out = hcu._C.sparse_mask_topk_transform_split_pre(x.to(dev), mask.to(dev), lens.to(dev), pt.to(dev), cu, 2048,
                                                      8, torch.from_numpy(zws).to(dev))
    assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("dist", ["relu_sum", "ties", "sparse2", "const"])
def test_topk_keys_sorted_order(hcu, dev, dist):
    x, mask, lens, pt = make_scores(4, 9000, dist, W=9000, ragged=True, seed=13)
    ref, rkeys = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy(), return_keys=True)
    idx, keys = hcu.topk_keys(x.to(dev), mask.to(dev), lens.to(dev), pt.to(dev))
    idx, keys = idx.cpu().numpy(), keys.cpu().numpy().view(np.uint32)
    for r in range(4):
        v = ref[r] >= 0
        order = np.argsort(ref[r][v], kind="stable")
        assert np.array_equal(idx[r][v], ref[r][v][order])
        assert np.array_equal(keys[r][v], rkeys[r][v][order])
        assert (idx[r][~v] == -1).all()


def test_topk_rows_and_empty_batch(hcu, dev):
    x, mask, lens, pt = make_scores(192, 16384, "relu_sum", W=16448, ragged=True, seed=17)
    ref = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy())
    out = hcu.sparse_mask_topk_transform(x.to(dev), mask.to(dev), lens.to(dev), pt.to(dev),
                                         torch.arange(193, dtype=torch.int32, device=dev))
    assert np.array_equal(out.cpu().numpy(), ref)
    e = torch.empty(0, 4096, device=dev)
    out = hcu.sparse_mask_topk_transform(e, torch.empty(0, 256, dtype=torch.int16, device=dev),
                                         torch.empty(0, dtype=torch.int32, device=dev),
                                         torch.empty(0, 4096, dtype=torch.int32, device=dev),
                                         torch.zeros(1, dtype=torch.int32, device=dev))
    assert tuple(out.shape) == (0, 2048)


def _adversarial_rows(W):
    """Rows aimed at the candidate path's limits: a sample-derived bound that misses (large
    values exactly at the sampled 4-token groups), candidates clustered at the row end, more
    tokens tied at the bound than the candidate list holds (8192 on the 1024-thread kernel,
    4096 on the 512-thread one used for rows up to 32K tokens), an all-negative row, a sparse
    row (threshold +0) and a short mixed-sign row.  Each must still equal the oracle exactly."""
    rng = np.random.default_rng(23)
    x = rng.random((6, W), dtype=np.float32)
    mask_bits = np.ones((6, W), dtype=bool)
    l2 = W * 5 // 8
    lens = np.array([W, W, l2, W // 2, W // 2, 5000], dtype=np.int32)
    groups = 512  # 2048 samples in groups of 4 consecutive tokens
    stride_g = np.float32(W) / np.float32(groups)
    start = ((np.arange(groups, dtype=np.float32) + np.float32(0.5)) * stride_g).astype(np.int64) & ~3
    start = np.minimum(start, (W - 4) & ~3)
    pos = (start[:, None] + np.arange(4)).reshape(-1)
    x[0, pos] = 1000.0 + rng.random(pos.size, dtype=np.float32)
    x[1] = np.arange(W, dtype=np.float32) + rng.random(W, dtype=np.float32)
    x[2, :l2] = rng.random(l2, dtype=np.float32) * 0.25
    x[2, rng.permutation(l2)[:1000]] = 2.0 + rng.random(1000, dtype=np.float32)
    tied = rng.permutation(l2)
    tied = tied[~np.isin(tied, np.flatnonzero(x[2] >= 2.0))][:9000 if W > 32768 else 5000]
    x[2, tied] = 0.5
    x[3] = -1.0 - rng.random(W, dtype=np.float32)
    mask_bits[4] = rng.random(W) < 0.05  # ~5 % positives: threshold +0 for the shorter rows
    x[5] = rng.standard_normal(W).astype(np.float32)
    x[~mask_bits] = np.nan
    mask = O.pack_mask(mask_bits)
    pt = np.stack([rng.permutation(W).astype(np.int32) for _ in range(6)])
    return torch.from_numpy(x), torch.from_numpy(mask), torch.from_numpy(lens), torch.from_numpy(pt)


@pytest.mark.parametrize("W", [65536, 32768])
def test_topk_candidate_bound_edge_cases(hcu, dev, W):
    x, mask, lens, pt = _adversarial_rows(W)
    assert np.array_equal(O.mask_bits(mask.numpy(), W), ~np.isnan(x.numpy()))
    ref, rkeys = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy(), return_keys=True)
    for name, out in _run_all(hcu, x, mask, lens, pt, dev).items():
        assert np.array_equal(out.cpu().numpy(), ref), name
    ident = torch.arange(W, dtype=torch.int32).repeat(6, 1)
    refi = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), ident.numpy())
    idx, keys = hcu.topk_keys(x.to(dev), mask.to(dev), lens.to(dev), ident.to(dev))
    idx = idx.cpu().numpy()
    for r in range(6):
        v = refi[r] >= 0
        assert np.array_equal(idx[r][v], np.sort(refi[r][v])), r
