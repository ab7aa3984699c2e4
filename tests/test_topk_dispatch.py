"""CPU check of which top-k strategy hcu_ops.sparse_mask_topk_transform picks (no GPU: the _C entry
points are replaced by recorders and the SM count is fixed at 148).  At least two rows per SM with
widths in (8192, 131072] go through the per-row candidate lists; fewer rows, narrower or wider rows
keep the block-per-row kernel (through the split entry, as the reference's default switch does);
HCU_TOPK_LISTS=0 turns the list strategy off; a pass-1 histogram built for the same scores and
lengths is consumed first."""
import types

import pytest
import torch


@pytest.fixture
def ops(monkeypatch):
    import hcu_ops

    calls = []

    def rec(name):
        return lambda *a, **k: calls.append(name) or name

    fake = types.SimpleNamespace(**{n: rec(n) for n in (
        "sparse_mask_topk_transform", "sparse_mask_topk_transform_split", "sparse_mask_topk_transform_split_pre",
        "sparse_mask_topk_transform_lists")})
    monkeypatch.setattr(hcu_ops, "_C", fake)
    monkeypatch.setattr(hcu_ops, "_N_CU", 148)
    monkeypatch.setattr(hcu_ops, "_MQA_HIST", None)
    return hcu_ops, calls


def _call(hcu, rows, width, lengths=None):
    score = torch.empty(1).expand(rows, width)  # the shape only; no memory behind it
    lengths = torch.zeros(rows, dtype=torch.int32) if lengths is None else lengths
    return hcu.sparse_mask_topk_transform(score, None, lengths, None, None, 2048), score, lengths


@pytest.mark.parametrize("rows,width,expect", [
    (296, 65536, "sparse_mask_topk_transform_lists"),     # two rows per SM
    (8192, 73728, "sparse_mask_topk_transform_lists"),    # prefill chunk
    (16384, 131072, "sparse_mask_topk_transform_lists"),  # the widest the lists' select covers
    (295, 65536, "sparse_mask_topk_transform_split"),     # fewer rows: one CTA (or cluster) per row
    (8192, 8192, "sparse_mask_topk_transform_split"),     # narrow rows
    (8192, 131088, "sparse_mask_topk_transform_split"),   # past the select's width
    (128, 65536, "sparse_mask_topk_transform_split"),     # the decode shape
])
def test_strategy_by_shape(ops, rows, width, expect):
    hcu, calls = ops
    _call(hcu, rows, width)
    assert calls == [expect]


def test_lists_switch_off(ops, monkeypatch):
    hcu, calls = ops
    monkeypatch.setattr(hcu, "_TOPK_LISTS", False)
    _call(hcu, 8192, 73728)
    assert calls == ["sparse_mask_topk_transform_split"]


def test_histogram_hand_off_comes_first(ops, monkeypatch):
    hcu, calls = ops
    score = torch.empty(1).expand(8192, 73728)
    lengths = torch.zeros(8192, dtype=torch.int32)
    monkeypatch.setattr(hcu, "_MQA_HIST", (score, lengths, None))
    hcu.sparse_mask_topk_transform(score, None, lengths, None, None, 2048)
    assert calls == ["sparse_mask_topk_transform_split_pre"]
    assert hcu._MQA_HIST is None
