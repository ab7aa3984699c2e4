"""GPU parity of the indexer-K cache writer (quantise per token -> fp8 e4m3 + fp32 scale pages):
bit-exact against the oracle for fp32 and bf16 rows, untouched slots preserved, out-of-range slots
skipped and flagged, and the written cache read back by the dequant and logits ops."""
import numpy as np
import pytest
import torch

from indexer_testlib import compare_logits
from oracle import indexer as O

pytestmark = pytest.mark.gpu


def _rows(n, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(max(n, 5), 128, generator=g) * 2.0
    k[0] = 0.0                                     # amax 0: the clamped scale
    k[1] = torch.randn(128, generator=g) * 1e-30   # subnormal-range values
    k[2, 7] = 3.0e38                               # one value near fp32 max, the rest flush to 0
    k[3] = -k[3].abs()                             # all negative
    k[4] = 1.0                                     # all equal
    return k[:n].to(dtype) if n >= 5 else k[[0, 2, 4, 1, 3][:n]].to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [1, 5, 333, 4096])
def test_kstore_bit_exact(hcu, dev, dtype, n):
    n_pages = (n + 63) // 64 + 7
    k = _rows(n, seed=n, dtype=dtype)
    g = torch.Generator().manual_seed(100 + n)
    loc = torch.randperm(n_pages * 64, generator=g)[:n].to(torch.int32)
    pool0 = torch.randint(0, 256, (n_pages, 64, 1, 132), generator=g, dtype=torch.uint8)  # stale bytes
    ref = O.quant_store_index_k(k.float().numpy(), loc.numpy(), pool0.view(n_pages, -1).numpy())
    pool = pool0.to(dev)
    out = hcu.quant_store_index_k(k.to(dev), loc.to(dev), pool)
    assert out.data_ptr() == pool.data_ptr()
    assert np.array_equal(pool.view(n_pages, -1).cpu().numpy(), ref)


def _midpoint_rows(n_rows, seed):
    """fp32 rows whose quotients x / scale sit on and beside the rounding midpoints of fp8 e4m3:
    per row an awkward amax (so an inexact scale), then x = fl(m * scale) and its two fp32
    neighbours for midpoints m between consecutive e4m3 values, both signs."""
    rng = np.random.default_rng(seed)
    e4 = torch.arange(0, 127, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    mids = ((e4[:-1] + e4[1:]) / 2)
    mids = mids[mids < 440.0].astype(np.float32)
    rows = np.zeros((n_rows, 128), np.float32)
    for r in range(n_rows):
        amax = np.float32(rng.uniform(0.5, 2.0) * 2.0 ** rng.integers(-30, 40))
        scale = np.float32(np.maximum(amax, np.float32(1e-12)) / np.float32(448.0))
        m = rng.choice(mids, 42) * rng.choice(np.array([-1.0, 1.0], np.float32), 42)
        x = (m.astype(np.float32) * scale).astype(np.float32)
        v = np.concatenate([x, np.nextafter(x, np.float32(np.inf)), np.nextafter(x, np.float32(-np.inf))])
        rows[r, 0] = amax
        rows[r, 1:127] = v[:126]
        rows[r, 127] = -amax
    return torch.from_numpy(rows)


@pytest.mark.parametrize("kind", ["midpoints", "wide_exponents"])
def test_kstore_division_edges(hcu, dev, kind):
    """The quotient x / scale is formed from one reciprocal per token and an FMA correction: bit
    equal to the oracle's IEEE division on values at and beside every e4m3 rounding midpoint, and on
    values spread over 2^-60 .. 2^60 within a row."""
    n = 2048
    if kind == "midpoints":
        k = _midpoint_rows(n, seed=5)
    else:
        g = torch.Generator().manual_seed(6)
        k = torch.randn(n, 128, generator=g) * torch.exp2(torch.randint(-60, 61, (n, 128), generator=g).float())
    n_pages = n // 64
    loc = torch.arange(n, dtype=torch.int32)
    ref = O.quant_store_index_k(k.numpy(), loc.numpy(), np.zeros((n_pages, 64 * 132), np.uint8))
    pool = torch.zeros(n_pages, 64, 1, 132, dtype=torch.uint8, device=dev)
    hcu.quant_store_index_k(k.to(dev), loc.to(dev), pool)
    assert np.array_equal(pool.view(n_pages, -1).cpu().numpy(), ref)


def test_kstore_strided_rows(hcu, dev):
    n, n_pages = 200, 8
    big = _rows(n, seed=9, dtype=torch.float32)
    wide = torch.zeros(n, 192)
    wide[:, :128] = big
    k = wide.to(dev)[:, :128]  # row stride 192 elements
    loc = torch.arange(n, dtype=torch.int32)
    ref = O.quant_store_index_k(big.numpy(), loc.numpy(), np.zeros((n_pages, 64 * 132), np.uint8))
    pool = torch.zeros(n_pages, 64, 1, 132, dtype=torch.uint8, device=dev)
    hcu.quant_store_index_k(k, loc.to(dev), pool)
    assert np.array_equal(pool.view(n_pages, -1).cpu().numpy(), ref)


def test_kstore_out_of_range_slot_is_skipped_and_flagged(hcu, dev, request):
    request.node.allowed_status = 2  # HCU_STATUS_BAD_INPUT
    n_pages = 2
    k = _rows(6, seed=4, dtype=torch.float32)
    loc = torch.tensor([0, -1, 5, n_pages * 64, 127, 64], dtype=torch.int32)
    pool = torch.full((n_pages, 64, 1, 132), 0xAB, dtype=torch.uint8, device=dev)
    ref = O.quant_store_index_k(k.numpy(), loc.numpy(), pool.view(n_pages, -1).cpu().numpy())
    hcu.quant_store_index_k(k.to(dev), loc.to(dev), pool)
    st = hcu.read_device_status(clear=False)
    assert st & 2
    assert np.array_equal(pool.view(n_pages, -1).cpu().numpy(), ref)


def test_kstore_then_dequant_and_logits(hcu, dev):
    """Write a decode workload's K through the writer, then read it with dequant_index_k_paged and
    mqa_logits: same results as the oracle on the oracle-written cache."""
    from hcu_ops.workloads import make_decode

    w = make_decode(3, 2, [5000, 777, 3000], heads=64, seed=12, extra_pages=4)
    n_pages = w["kv_cache"].shape[0]
    g = torch.Generator().manual_seed(12)
    k = torch.randn(n_pages * 64, 128, generator=g).to(torch.bfloat16)
    loc = torch.randperm(n_pages * 64, generator=g).to(torch.int32)
    ref_pool = O.quant_store_index_k(k.float().numpy(), loc.numpy(), np.zeros((n_pages, 64 * 132), np.uint8))
    pool = torch.zeros(n_pages, 64, 1, 132, dtype=torch.uint8, device=dev)
    hcu.quant_store_index_k(k.to(dev), loc.to(dev), pool)
    assert np.array_equal(pool.view(n_pages, -1).cpu().numpy(), ref_pool)
    # dequant of the written slots
    sel = loc[:1000].to(dev)
    got = hcu.dequant_index_k_paged(pool, sel).view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, O.dequant_index_k(ref_pool, loc[:1000].numpy()))
    # logits over the written cache
    d = {kk: (v.to(dev) if torch.is_tensor(v) else v) for kk, v in w.items()}
    lg, mk, _ = hcu._C.mqa_logits_hist(d["q"], pool, d["weights"], d["context_lens"], d["block_table"],
                                       d["max_context_len"], d["group_size"], 0, 0, None)
    rl, rm, fl = O.mqa_logits_paged(w["q"].view(torch.uint8).numpy().reshape(w["q"].shape[0], 64, 128), ref_pool,
                                    w["weights"].numpy(), w["context_lens"].numpy(), w["block_table"].numpy(),
                                    w["max_context_len"], w["group_size"], want_floor=True)
    res = compare_logits(lg.cpu().numpy(), mk.cpu().numpy(), rl, rm, fl)
    assert res["ok"], res
