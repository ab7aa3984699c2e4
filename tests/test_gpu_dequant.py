"""GPU parity of stage 1 (paged K-cache dequant): bit-exact against the oracle."""
import numpy as np
import pytest
import torch

from indexer_testlib import golden
from oracle import indexer as O

pytestmark = pytest.mark.gpu


def test_mla_dequant_matches_reference_triton_fixture(hcu, dev):
    g = golden("dequant_mla_triton.npz")
    cache = torch.from_numpy(g["cache"]).to(dev)
    page = torch.from_numpy(g["page"]).to(dev)
    out = hcu.dequantize_k_cache_paged(cache, page)
    assert out.shape == (page.shape[0], 1, 576) and out.dtype == torch.bfloat16
    assert np.array_equal(out.view(torch.int16).cpu().numpy().reshape(page.shape[0], -1),
                          g["out_bits"].reshape(page.shape[0], -1))


@pytest.mark.parametrize("n_tokens,pool", [(1, 7), (29, 40), (5000, 3000), (131072, 65536)])
def test_mla_dequant_bitexact(hcu, dev, n_tokens, pool):
    from hcu_ops.workloads import make_mla_dequant

    w = make_mla_dequant(n_tokens, pool, seed=n_tokens)
    out = hcu.dequantize_k_cache_paged(w["quant_k_cache"].to(dev), w["page_table_1_flattened"].to(dev))
    ref = O.dequant_mla_656(w["quant_k_cache"].view(torch.uint8).numpy().reshape(pool, 656),
                            w["page_table_1_flattened"].numpy())
    got = out.view(torch.int16).cpu().numpy().reshape(n_tokens, 576).view(np.uint16)
    assert np.array_equal(got, ref)


def test_mla_dequant_special_values(hcu, dev):
    """NaN / inf / subnormal scales and fp8 NaN bytes: one RNE conversion, canonical NaN."""
    rng = np.random.default_rng(11)
    pool = 64
    cache = rng.integers(0, 256, (pool, 656), dtype=np.uint8)  # every fp8 byte incl. 0x7f/0xff NaN
    sc = np.array([np.inf, -np.inf, np.nan, 1e-40, -1e-42, 3.4e38, 1.0, -0.0], np.float32)
    cache[:, 512:528] = rng.choice(sc, (pool, 4)).astype(np.float32).view(np.uint8).reshape(pool, 16)
    page = rng.integers(0, pool, 300).astype(np.int32)
    out = hcu.dequantize_k_cache_paged(torch.from_numpy(cache).to(dev), torch.from_numpy(page).to(dev))
    ref = O.dequant_mla_656(cache, page)
    got = out.view(torch.int16).cpu().numpy().reshape(300, 576).view(np.uint16)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("n_tokens,pool_pages", [(1, 3), (64, 2), (1000, 40), (131072, 4096)])
def test_index_k_dequant_bitexact(hcu, dev, n_tokens, pool_pages):
    from hcu_ops.workloads import make_index_k_dequant

    w = make_index_k_dequant(n_tokens, pool_pages, seed=2)
    out = hcu.dequant_index_k_paged(w["kv_cache"].to(dev), w["token_loc"].to(dev))
    ref = O.dequant_index_k(w["kv_cache"].numpy().reshape(pool_pages, -1), w["token_loc"].numpy())
    assert np.array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), ref)


def test_dequant_out_of_range_slot_is_skipped_and_flagged(hcu, dev, request):
    request.node.allowed_status = 2  # HCU_STATUS_BAD_INPUT
    from hcu_ops.workloads import make_mla_dequant

    w = make_mla_dequant(8, 16, seed=5)
    page = w["page_table_1_flattened"].clone()
    page[3] = 16  # one past the pool
    page[5] = -1
    out_init = torch.full((8, 1, 576), 7.0, dtype=torch.bfloat16, device=dev)
    out = hcu.dequantize_k_cache_paged(w["quant_k_cache"].to(dev), page.to(dev))
    del out_init
    st = hcu.read_device_status(clear=False)
    assert st & 2
    good = [i for i in range(8) if i not in (3, 5)]
    ref = O.dequant_mla_656(w["quant_k_cache"].view(torch.uint8).numpy().reshape(16, 656), page.numpy()[good])
    got = out.view(torch.int16).cpu().numpy().reshape(8, 576).view(np.uint16)[good]
    assert np.array_equal(got, ref)
