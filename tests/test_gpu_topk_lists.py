"""GPU parity of the list top-k for many rows (hcu_sparse_mask_topk_transform_lists: a warp per row
derives a sampled bound, a warp per row streams the row into a candidate list, the list select
writes the canonical order, the block-per-row kernel rewrites per row whatever a list could not
prove): bit for bit, order included, equal to the plain top-k and to the oracle on the
reference's ten score distributions (``hcu_ops/tests/topk_lib.py:8-51`` of the reference,
restated in indexer_testlib.make_scores), at lengths listed whole (<= 4096), bounded lengths up to
the 131072 maximum, ragged rows, an unaligned row stride (scalar loads), distributions whose lists
overflow or miss (per-row exact rewrite), many rows, graph replay, and the prefill logits of the
ragged kernel."""
import numpy as np
import pytest
import torch

from indexer_testlib import DISTS, make_scores, same_values
from oracle import indexer as O

pytestmark = pytest.mark.gpu


def _both(hcu, x, mask, lens, pt, dev):
    xs, ms, ls, ps = (t.to(dev) for t in (x, mask, lens, pt))
    cu = torch.arange(x.shape[0] + 1, dtype=torch.int32, device=dev)
    return (hcu._C.sparse_mask_topk_transform_lists(xs, ms, ls, ps, cu, 2048),
            hcu._C.sparse_mask_topk_transform(xs, ms, ls, ps, cu, 2048))


@pytest.mark.parametrize("dist", DISTS)
@pytest.mark.parametrize("L", [3000, 9000, 40000, 70000, 131072])
@pytest.mark.parametrize("ragged", [False, True])
def test_lists_equal_plain_and_oracle(hcu, dev, dist, L, ragged):
    W = min(L + 64, 131072)
    x, mask, lens, pt = make_scores(6, L, dist, W=W, ragged=ragged, seed=L + 7)
    got, plain = _both(hcu, x, mask, lens, pt, dev)
    assert torch.equal(got, plain), (dist, L, ragged)
    ref = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy())
    out = got.cpu().numpy()
    assert np.array_equal(out, ref), (dist, L, ragged)
    assert same_values(x.numpy(), lens.numpy(), ref, out, pt.numpy())


@pytest.mark.parametrize("dist", ["relu_sum", "ties", "mixed"])
def test_lists_unaligned_stride(hcu, dev, dist):
    """A row stride that is not a multiple of 4 floats: the scalar-load instances."""
    L, W = 50000, 50003
    x, mask, lens, pt = make_scores(5, L, dist, W=W, ragged=True, seed=9)
    got, plain = _both(hcu, x, mask, lens, pt, dev)
    assert torch.equal(got, plain)
    assert np.array_equal(got.cpu().numpy(), O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy()))


def test_lists_many_rows_mixed(hcu, dev):
    """400 rows from 1000 to 73728 tokens, then a call where some rows' lists overflow (constant
    rows among random ones: only those rows take the exact path), then the first call again."""
    B, W = 400, 73728
    x, mask, _, pt = make_scores(B, W, "relu_sum", W=W, seed=21)
    lens = torch.linspace(1000, W, B).to(torch.int32)
    got, plain = _both(hcu, x, mask, lens, pt, dev)
    assert torch.equal(got, plain)
    rows = [0, 17, 120, 250, B - 1]
    ref = O.topk_transform(x.numpy()[rows], mask.numpy()[rows], lens.numpy()[rows], pt.numpy()[rows])
    assert np.array_equal(got.cpu().numpy()[rows], ref)
    xc, mc, _, _ = make_scores(B, W, "const", W=W, seed=2)
    x2, m2 = x.clone(), mask.clone()
    x2[::7], m2[::7] = xc[::7], mc[::7]
    got, plain = _both(hcu, x2, m2, lens, pt, dev)
    assert torch.equal(got, plain)
    got, plain = _both(hcu, x, mask, lens, pt, dev)
    assert torch.equal(got, plain)


def test_lists_graph_replay(hcu, dev):
    """Captured once, replayed over new scores and lengths copied into the captured buffers."""
    B, W = 320, 40000
    x, mask, lens, pt = (t.to(dev) for t in make_scores(B, W, "relu_sum", W=W, ragged=True, seed=1))
    cu = torch.arange(B + 1, dtype=torch.int32, device=dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        hcu._C.sparse_mask_topk_transform_lists(x, mask, lens, pt, cu, 2048)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = hcu._C.sparse_mask_topk_transform_lists(x, mask, lens, pt, cu, 2048)
    for seed, dist in ((2, "mixed"), (3, "const"), (4, "relu_sum")):
        x2, m2, _, _ = make_scores(B, W, dist, W=W, seed=seed)
        l2 = torch.randint(100, W + 1, (B,), generator=torch.Generator().manual_seed(seed)).to(torch.int32)
        x.copy_(x2.to(dev))
        mask.copy_(m2.to(dev))
        lens.copy_(l2.to(dev))
        g.replay()
        assert torch.equal(out, hcu._C.sparse_mask_topk_transform(x, mask, lens, pt, cu, 2048)), dist


def test_lists_rejects_wide_rows(hcu, dev):
    x, mask, lens, pt = (t.to(dev) for t in make_scores(1, 4096, "pos", W=131072 + 16))
    cu = torch.arange(2, dtype=torch.int32, device=dev)
    with pytest.raises(RuntimeError):
        hcu._C.sparse_mask_topk_transform_lists(x, mask, lens, pt, cu, 2048)


def test_lists_on_prefill_logits(hcu, dev):
    """The ragged kernel's own logits (prefill shape, 512 rows past a 60000-token prefix), through
    the wrapper's dispatch as well."""
    from hcu_ops.workloads import make_ragged

    d = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in make_ragged(512, 60000, heads=64, seed=4).items()}
    lg, mk = hcu.mqa_logits_ragged(d["q"], d["k_fp8"], d["k_scale"], d["weights"], torch.zeros_like(d["row_end"]),
                                   d["row_end"])
    n = d["k_fp8"].shape[0]
    pt = torch.arange(n, dtype=torch.int32, device=dev).expand(512, n)
    cu = torch.arange(513, dtype=torch.int32, device=dev)
    args = (lg, mk, d["row_end"], pt, cu, 2048)
    plain = hcu._C.sparse_mask_topk_transform(*args)
    assert torch.equal(hcu._C.sparse_mask_topk_transform_lists(*args), plain)
    assert torch.equal(hcu.sparse_mask_topk_transform(*args), plain)
