"""GPU parity of the fused prefill indexer (hcu_ops.mqa_topk_ragged): its result equals the
materialising pair -- mqa_logits_ragged from token 0, then sparse_mask_topk_transform with
lengths = row_end -- bit for bit, order included, and that pair is itself checked against the
CPU oracle (test_gpu_prefill.py).  Cases: short rows (identity), rows listed whole, long rows
through the sampled bound, a row set that spans partial sample tiles, 32 heads, a permuted page
table, a bound forced above the threshold (the exact path runs and the result is unchanged), and
the benchmark's prefill shape on a row subset."""
import numpy as np
import pytest
import torch

from oracle import indexer as O

pytestmark = pytest.mark.gpu


def _unfused(hcu, d, pt):
    lg, mk = hcu.mqa_logits_ragged(d["q"], d["k_fp8"], d["k_scale"], d["weights"], torch.zeros_like(d["row_end"]),
                                   d["row_end"])
    cu = torch.arange(d["q"].shape[0] + 1, dtype=torch.int32, device=d["q"].device)
    return hcu.sparse_mask_topk_transform(lg, mk, d["row_end"], pt, cu, 2048), lg, mk


def _dev(w, dev):
    return {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in w.items()}


def _ident(d):
    n = d["k_fp8"].shape[0]
    return torch.arange(n, dtype=torch.int32, device=d["q"].device).expand(d["q"].shape[0], n)


CASES = [
    # rows, prefix, heads, n_tokens
    (40, 0, 64, None),         # rows of 1..40 tokens: identity rows only
    (24, 3000, 64, None),      # 3001..3024 tokens: every visible token listed (rows <= 8192)
    (33, 20000, 64, None),     # sampled bound; a ragged last super-block
    (16, 60000, 32, None),     # 32 heads
    (48, 9000, 64, 12000),     # K past every row's end; row ends inside sample tiles
]


@pytest.mark.parametrize("case", CASES, ids=[f"r{c[0]}p{c[1]}h{c[2]}" for c in CASES])
def test_fused_equals_materialised(hcu, dev, case):
    from hcu_ops.workloads import make_ragged

    rows, prefix, heads, n_tok = case
    d = _dev(make_ragged(rows, prefix, heads=heads, seed=rows + prefix, n_tokens=n_tok), dev)
    pt = _ident(d)
    ref, _, _ = _unfused(hcu, d, pt)
    flag = torch.full((1,), 7, dtype=torch.int32, device=dev)
    got = hcu.mqa_topk_ragged(d["q"], d["k_fp8"], d["k_scale"], d["weights"], d["row_end"], pt, fallback_flag=flag)
    assert torch.equal(got, ref)
    assert int(flag.item()) == 0  # the lists proved exactness on their own
    assert hcu.read_device_status(clear=True) == 0


def test_fused_page_table_and_oracle(hcu, dev):
    """A permuted page table per row; the selected tokens also match the oracle's top-k of the
    device's own logits."""
    from hcu_ops.workloads import make_ragged

    rows, prefix = 20, 30000
    d = _dev(make_ragged(rows, prefix, heads=64, seed=11), dev)
    n = d["k_fp8"].shape[0]
    g = torch.Generator().manual_seed(3)
    pt = torch.stack([torch.randperm(n, generator=g) for _ in range(rows)]).to(torch.int32).to(dev)
    ref, lg, mk = _unfused(hcu, d, pt)
    got = hcu.mqa_topk_ragged(d["q"], d["k_fp8"], d["k_scale"], d["weights"], d["row_end"], pt)
    assert torch.equal(got, ref)
    o = O.topk_transform(lg.cpu().numpy(), mk.cpu().numpy(), d["row_end"].cpu().numpy(), pt.cpu().numpy())
    assert np.array_equal(got.cpu().numpy(), o)


def test_fused_bound_above_threshold_takes_exact_path(hcu, dev):
    """K rows of the sampled tiles scaled up (their scores dominate the sample), so the sampled
    bound lies above the rows' true top-2048 threshold and the lists hold fewer than 2048 tokens:
    the select raises the flag, the predicated exact path rewrites every row, and the result still
    equals the materialising pair's."""
    from hcu_ops.workloads import make_ragged

    rows, prefix = 12, 40000
    w = make_ragged(rows, prefix, heads=64, seed=21)
    n = w["k_fp8"].shape[0]
    tile = torch.arange(n) // 128
    sampled = (tile % 64) == 32  # the tiles the fused path samples (one in 64, at offset 32)
    ks = w["k_scale"].clone()
    ks[sampled] *= 64.0
    w["k_scale"] = ks
    d = _dev(w, dev)
    pt = _ident(d)
    ref, _, _ = _unfused(hcu, d, pt)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    got = hcu.mqa_topk_ragged(d["q"], d["k_fp8"], d["k_scale"], d["weights"], d["row_end"], pt, fallback_flag=flag)
    assert int(flag.item()) == 1
    assert torch.equal(got, ref)
    # the next call on ordinary inputs clears the flag again
    d2 = _dev(make_ragged(rows, prefix, heads=64, seed=22), dev)
    ref2, _, _ = _unfused(hcu, d2, pt)
    got2 = hcu.mqa_topk_ragged(d2["q"], d2["k_fp8"], d2["k_scale"], d2["weights"], d2["row_end"], pt,
                               fallback_flag=flag)
    assert int(flag.item()) == 0
    assert torch.equal(got2, ref2)


def test_fused_graph_replay(hcu, dev):
    """Captured in a CUDA graph and replayed over new inputs copied into the captured buffers."""
    from hcu_ops.workloads import make_ragged

    rows, prefix = 32, 16000
    d = _dev(make_ragged(rows, prefix, heads=64, seed=31), dev)
    pt = _ident(d)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        hcu.mqa_topk_ragged(d["q"], d["k_fp8"], d["k_scale"], d["weights"], d["row_end"], pt)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = hcu.mqa_topk_ragged(d["q"], d["k_fp8"], d["k_scale"], d["weights"], d["row_end"], pt)
    for seed in (32, 33):
        d2 = _dev(make_ragged(rows, prefix, heads=64, seed=seed), dev)
        for k in ("q", "k_fp8", "k_scale", "weights", "row_end"):
            d[k].copy_(d2[k])
        g.replay()
        ref, _, _ = _unfused(hcu, d, pt)
        assert torch.equal(out, ref)


@pytest.mark.slow
def test_fused_benchmark_prefill_shape(hcu, dev):
    """The benchmark's prefill shape (8192 rows x (65536 + i + 1) tokens) on its first 1024 rows,
    which keep the full 65.5K-73.7K-token K: equal to the materialising pair."""
    from hcu_ops.workloads import make_ragged

    w = make_ragged(8192, 65536, heads=64, seed=0)
    sel = slice(0, 1024)
    d = _dev({"q": w["q"][sel].contiguous(), "k_fp8": w["k_fp8"], "k_scale": w["k_scale"],
              "weights": w["weights"][sel].contiguous(), "row_end": w["row_end"][sel].contiguous()}, dev)
    pt = _ident(d)
    ref, _, _ = _unfused(hcu, d, pt)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    got = hcu.mqa_topk_ragged(d["q"], d["k_fp8"], d["k_scale"], d["weights"], d["row_end"], pt, fallback_flag=flag)
    assert int(flag.item()) == 0
    assert torch.equal(got, ref)
