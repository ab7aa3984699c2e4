"""GPU parity of stage 2 (paged MQA logits on tcgen05) and of the decode pipeline.

Logits: within the build's tolerance of the oracle (``indexer_testlib.compare_logits``);
masks identical except at values indistinguishable from zero.  Pass-1 workspace: exact
against the oracle on the device's own logits.  Top-k on the device's logits: exact.
End to end: >= 99.9% overlap with the oracle's own selection."""
import numpy as np
import pytest
import torch

from indexer_testlib import compare_logits, overlap
from oracle import indexer as O

pytestmark = pytest.mark.gpu


def _decode(reqs, next_n, lens, heads, seed=0, width_pages=None):
    from hcu_ops.workloads import make_decode

    return make_decode(reqs, next_n, lens, heads=heads, seed=seed, width_pages=width_pages, extra_pages=3)


def _oracle_logits(w):
    return O.mqa_logits_paged(w["q"].view(torch.uint8).numpy().reshape(w["q"].shape[0], w["heads"], 128),
                              w["kv_cache"].numpy().reshape(w["kv_cache"].shape[0], -1), w["weights"].numpy(),
                              w["context_lens"].numpy(), w["block_table"].numpy(), w["max_context_len"],
                              w["group_size"], want_floor=True)


def _device(w, dev):
    return {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in w.items()}


def _run(hcu, d, hist_lens=None):
    return hcu._C.mqa_logits_hist(d["q"], d["kv_cache"], d["weights"], d["context_lens"], d["block_table"],
                                  d["max_context_len"], d["group_size"], 0, 0, hist_lens)


CASES = [
    # (reqs, next_n, per-request lengths, heads)
    (1, 1, [8192], 64),                      # config 0
    (1, 1, [8192], 32),                      # reference head count
    (4, 2, [5000, 130, 64, 4097], 64),       # MTP verify pairs
    (2, 6, [3000, 700], 32),                 # reference G=6
    (2, 6, [3000, 700], 64),                 # G=6 with 64 heads: two row blocks per group
    (3, 1, [1, 15, 16], 64),
    (3, 1, [63, 64, 65], 64),
    (3, 1, [127, 128, 129], 32),
    (3, 1, [2047, 2048, 2049], 64),
]


@pytest.mark.parametrize("case", CASES, ids=[f"r{c[0]}g{c[1]}h{c[3]}_{c[2][0]}" for c in CASES])
def test_logits_vs_oracle(hcu, dev, case):
    reqs, next_n, lens, heads = case
    w = _decode(reqs, next_n, lens, heads, seed=len(lens) + heads)
    d = _device(w, dev)
    lg, mk, zws = _run(hcu, d)
    rl, rm, fl = _oracle_logits(w)
    res = compare_logits(lg.cpu().numpy(), mk.cpu().numpy(), rl, rm, fl)
    assert res["ok"], res
    assert res["n_set"] > 0


def test_logits_nan_inputs_follow_fmaxf(hcu, dev):
    """NaN fp8 bytes (e4m3fn 0x7F / 0xFF) in the K pages and in q: the reference's ReLU is fmaxf,
    so a NaN dot product contributes 0 and every stored logit is finite."""
    w = _decode(2, 2, [3000, 1500], 64, seed=21)
    kv = w["kv_cache"].view(w["kv_cache"].shape[0], -1)
    page = int(w["block_table"][0, 0])
    kv[page, 5 * 128:6 * 128] = 0x7F       # token 5 of request 0: every byte NaN
    kv[page, 20 * 128 + 3] = 0xFF          # token 20: one negative-NaN byte
    qb = w["q"].view(torch.uint8).view(w["q"].shape[0], w["heads"], 128)
    qb[1, 9, 0] = 0x7F                     # one head of row 1
    lg, mk, _ = _run(hcu, _device(w, dev))
    rl, rm, fl = _oracle_logits(w)
    res = compare_logits(lg.cpu().numpy(), mk.cpu().numpy(), rl, rm, fl)
    assert res["ok"], res
    got = lg.cpu().numpy()
    assert np.isfinite(got[O.mask_bits(mk.cpu().numpy(), got.shape[1])]).all()


def test_logits_zero_length_rows_and_padded_table(hcu, dev):
    w = _decode(3, 1, [200, 300, 100], 64, seed=3, width_pages=64)
    w["context_lens"][1] = 0
    d = _device(w, dev)
    lg, mk, _ = _run(hcu, d)
    rl, rm, fl = _oracle_logits(w)
    res = compare_logits(lg.cpu().numpy(), mk.cpu().numpy(), rl, rm, fl)
    assert res["ok"], res
    assert (mk[1] == 0).all()


@pytest.mark.parametrize("next_n,heads", [(2, 64), (1, 64), (4, 64), (2, 32)])
def test_logits_many_items_per_cta(hcu, dev, next_n, heads):
    """Long contexts: every CTA streams dozens of tiles, so the stage, TMEM-accumulator and
    Q rings wrap many times (rings of 8 or 10 stages against 4 producers and 3 teams)."""
    lens = [65536, 60000, 47000, 41000, 33333, 30000, 26000, 20001, 65536, 9000, 4096, 1]
    w = _decode(len(lens), next_n, lens, heads, seed=31)
    d = _device(w, dev)
    lg, mk, _ = _run(hcu, d)
    rl, rm, fl = _oracle_logits(w)
    res = compare_logits(lg.cpu().numpy(), mk.cpu().numpy(), rl, rm, fl)
    assert res["ok"], res


def test_hist_workspace_exact_on_device_logits(hcu, dev):
    w = _decode(4, 1, [9000, 2048, 2049, 30000], 64, seed=21)
    d = _device(w, dev)
    lens = d["context_lens"]
    lg, mk, zws = _run(hcu, d, hist_lens=lens)
    B, W = lg.shape
    g1, cnt = O.pass1_hist(lg.cpu().numpy(), mk.cpu().numpy(), lens.cpu().numpy(), W)
    z = zws.cpu().numpy()
    assert np.array_equal(z[: B * 4096].reshape(B, 4096), g1)
    assert not z[B * 4096: 2 * B * 4096].any()
    assert np.array_equal(z[2 * B * 4096:].reshape(B, 2), cnt)


@pytest.mark.parametrize("next_n,use_hist", [(2, False), (2, True), (1, True)])
def test_decode_pipeline(hcu, dev, next_n, use_hist):
    """mqa_logits -> sparse_mask_topk_transform as sglang calls them.  The fused pass-1
    histogram is taken for single rows up to HCU_MQA_HIST_MAX_ROWS (8) rows and, as in the
    reference, not for grouped rows (HCU_MQA_HIST_MAX_ROWS_G6 = 0)."""
    w = _decode(3, next_n, [40000, 9000, 3000], 64, seed=5)
    d = _device(w, dev)
    lens = d["context_lens"]
    logits, mask = hcu.mqa_logits(d["q"].contiguous(), d["kv_cache"], d["weights"], lens, d["block_table"],
                                  d["max_context_len"], d["group_size"], hist_lens=lens if use_hist else None)
    assert (hcu._MQA_HIST is not None) == (use_hist and next_n == 1)
    out = hcu.sparse_mask_topk_transform(logits, mask, lens, d["page_table_size_1"], d["cu_seqlens_q"], 2048)
    assert hcu._MQA_HIST is None
    got = out.cpu().numpy()
    # exact on identical logits
    ref_same = O.topk_transform(logits.cpu().numpy(), mask.cpu().numpy(), lens.cpu().numpy(),
                                w["page_table_size_1"].numpy())
    assert np.array_equal(got, ref_same)
    # end to end against the oracle's own logits
    rl, rm, _ = _oracle_logits(w)
    ref_e2e = O.topk_transform(rl, rm, lens.cpu().numpy(), w["page_table_size_1"].numpy())
    assert overlap(got, ref_e2e) >= 0.999


def test_logits_cuda_graph_replay(hcu, dev):
    """The decode indexer is captured once and replayed with new lengths (no host syncs)."""
    w = _decode(2, 2, [6000, 3000], 64, seed=8, width_pages=128)
    d = _device(w, dev)
    lens = d["context_lens"]
    pt, cu = d["page_table_size_1"], d["cu_seqlens_q"]

    def step():
        lg, mk = hcu.mqa_logits(d["q"], d["kv_cache"], d["weights"], lens, d["block_table"], d["max_context_len"],
                                d["group_size"])
        return hcu.sparse_mask_topk_transform(lg, mk, lens, pt, cu, 2048)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = step()
    for new in ([6000, 3000], [2500, 7000], [100, 8000]):
        lens.copy_(torch.tensor([new[0] - 1, new[0], new[1] - 1, new[1]], dtype=torch.int32))
        g.replay()
        torch.cuda.synchronize()
        eager = step()
        assert torch.equal(out, eager), new
