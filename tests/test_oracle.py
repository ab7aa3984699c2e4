"""CPU tests of the oracle: pinned against the golden fixtures made from the reference's own code,
plus internal properties.  No GPU needed."""
import numpy as np
import pytest
import torch

from indexer_testlib import DISTS, golden, make_scores, same_values
from oracle import indexer as O


# --------------------------------------------------------------------------- pins
def test_dequant_pinned_to_reference_triton_kernel():
    """Oracle == the reference's Triton v2 dequant (interpreter, exact-product inputs), bit for bit."""
    g = golden("dequant_mla_triton.npz")
    out = O.dequant_mla_656(g["cache"].reshape(-1, 656), g["page"])
    assert np.array_equal(out.view(np.int16).reshape(g["out_bits"].shape[0], -1),
                          g["out_bits"].reshape(g["out_bits"].shape[0], -1))


def test_pass1_hist_pinned_to_reference_ref_hist():
    """Oracle pass-1 histogram == the reference's torch ref_hist on the reference's generator."""
    g = golden("ref_hist_cases.npz")
    width = int(g["width"])
    for i in range(int(g["n"])):
        g1, cnt = O.pass1_hist(g[f"h{i}_x"], g[f"h{i}_mask"], g[f"h{i}_lens"], width)
        assert np.array_equal(g1, g[f"h{i}_g1"]), i
        assert np.array_equal(cnt, g[f"h{i}_cnt"]), i


def test_topk_on_reference_generator_cases():
    """Oracle top-k on the reference's own `make` outputs: the expected value multiset and the
    reference's validity criterion (unique, below length, -1 pads)."""
    g = golden("topk_make_cases.npz")
    for i in range(int(g["n"])):
        k = f"c{i:02d}"
        x, mask, lens, pt = g[f"{k}_x"], g[f"{k}_mask"], g[f"{k}_lengths"], g[f"{k}_pt"]
        out = O.topk_transform(x, mask, lens, pt)
        xv = np.nan_to_num(x, nan=0.0)
        idx = out.astype(np.int64) - pt[:, :1]
        vals = np.where(out >= 0, np.take_along_axis(xv, np.clip(idx, 0, x.shape[1] - 1), 1), -np.inf)
        assert np.array_equal(np.sort(vals, -1), g[f"{k}_sorted_values"]), k
        assert same_values(x, lens, out, out, pt), k


# --------------------------------------------------------------------------- properties
def test_bf16_rne_matches_torch_for_finite_values():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**32, 200000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x)]
    ours = O.f32_to_bf16_bits(x)
    ref = torch.from_numpy(x.copy()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, ref)
    assert O.f32_to_bf16_bits(np.array([np.nan], np.float32))[0] == 0x7FFF


def test_to_key_is_monotone():
    v = np.array([-np.inf, -3.0, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf], np.float32)
    k = O.to_key(v)
    assert (np.diff(k.astype(np.int64)) > 0).all()
    assert O.to_key(np.array([0.0], np.float32))[0] == 0x80000000


def test_mask_pack_roundtrip():
    rng = np.random.default_rng(1)
    bits = rng.random((3, 100)) < 0.4
    m = O.pack_mask(bits)
    assert m.shape == (3, 7) and m.dtype == np.int16
    assert np.array_equal(O.mask_bits(m, 100), bits)


@pytest.mark.parametrize("dist", DISTS)
def test_select_topk_matches_bruteforce(dist):
    x, mask, lens, pt = make_scores(3, 5000, dist, W=5100, ragged=True, seed=3)
    out, keys = O.topk_transform(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy(), return_keys=True)
    mb = O.mask_bits(mask.numpy(), 5100)
    for r in range(3):
        L = int(lens[r])
        k = O.row_keys(x.numpy()[r], mb[r], L)
        order = sorted(range(L), key=lambda i: (-int(k[i]), i))[:2048]
        got = out[r] - pt.numpy()[r, 0]
        assert set(got.tolist()) == set(order)
        thr = k[order[-1]]
        above = [i for i in order if k[i] > thr]
        ties = [i for i in order if k[i] == thr]
        assert got.tolist() == sorted(above) + sorted(ties)
        assert np.array_equal(keys[r], k[got])


def test_short_rows_select_everything_in_order():
    x, mask, lens, pt = make_scores(2, 700, "mixed", W=1000)
    out = O.topk_transform(x.numpy(), mask.numpy(), np.array([700, 0], np.int32), pt.numpy())
    assert out[0, :700].tolist() == pt.numpy()[0, :700].tolist()
    assert (out[0, 700:] == -1).all() and (out[1] == -1).all()


@pytest.mark.parametrize("parts", [2, 3, 8])
def test_cp_merge_equals_single_range(parts):
    rows, N = 5, 9000
    x, mask, _, _ = make_scores(rows, N, "relu_sum", W=N, seed=parts)
    xs, ms = x.numpy(), mask.numpy()
    vis = np.array([N, 3000, 2048, 100, 6001])
    ident = np.tile(np.arange(N, dtype=np.int32), (rows, 1))
    full = O.topk_transform(xs, ms, vis, ident)
    mb = O.mask_bits(ms, N)
    bounds = np.linspace(0, N, parts + 1).astype(int)
    keys = np.zeros((parts, rows, 2048), np.uint32)
    gidx = np.full((parts, rows, 2048), -1, np.int32)
    for p in range(parts):
        a, b = bounds[p], bounds[p + 1]
        for r in range(rows):
            L = max(0, min(b, vis[r]) - a)
            k = O.row_keys(xs[r, a:], mb[r, a:], L)
            sel = np.sort(O.select_topk(k))  # local lists in ascending token order
            keys[p, r, :sel.size] = k[sel]
            gidx[p, r, :sel.size] = sel + a
    merged = O.cp_merge(keys, gidx, vis)
    assert np.array_equal(merged, full)


def test_logits_oracle_matches_float64_definition():
    rng = np.random.default_rng(5)
    B, H, L = 2, 32, 200
    q = torch.from_numpy(rng.standard_normal((B, H, 128)).astype(np.float32)).to(torch.float8_e4m3fn)
    k = torch.from_numpy(rng.standard_normal((256, 128)).astype(np.float32)).to(torch.float8_e4m3fn)
    ks = rng.random(256).astype(np.float32) + 0.1
    w = rng.standard_normal((B, H)).astype(np.float32) / 8
    pages = np.concatenate([k.view(torch.uint8).numpy().reshape(4, 8192), ks.view(np.uint8).reshape(4, 256)], 1)
    perm = np.array([2, 0, 3, 1])
    kv = pages[np.argsort(perm)]  # logical page p lives at physical perm[p]
    bt = np.tile(perm.astype(np.int32), (B, 1))
    lens = np.array([L, 130], np.int32)
    lg, m, fl = O.mqa_logits_paged(q.view(torch.uint8).numpy(), kv, w, lens, bt, 256, 1, want_floor=True)
    qf = q.float().double().numpy()
    kf = k.float().double().numpy()
    for b in range(B):
        acc = qf[b] @ kf[: lens[b]].T
        s = (np.maximum(acc, 0) * w[b][:, None]).sum(0) * ks[: lens[b]]
        mb = O.mask_bits(m, 256)[b]
        assert mb[: lens[b]].all() and not mb[lens[b]:].any()
        assert np.allclose(lg[b, : lens[b]], s, rtol=1e-5, atol=1e-6)


def test_ragged_oracle_equals_paged_oracle():
    """Contiguous K with a per-row [0, end) range == the paged path with an identity block table."""
    rng = np.random.default_rng(7)
    R, H, N = 3, 64, 320
    q = torch.from_numpy(rng.standard_normal((R, H, 128)).astype(np.float32)).to(torch.float8_e4m3fn)
    k = torch.from_numpy(rng.standard_normal((N, 128)).astype(np.float32)).to(torch.float8_e4m3fn)
    ks = (rng.random(N).astype(np.float32) + 0.5) / 448
    w = rng.standard_normal((R, H)).astype(np.float32) / 8
    end = np.array([1, 200, 320], np.int32)
    lr, mr, _ = O.mqa_logits_ragged(q.view(torch.uint8).numpy(), k.view(torch.uint8).numpy(), ks, w,
                                    np.zeros(R, np.int32), end)
    pages = np.concatenate([k.view(torch.uint8).numpy().reshape(5, 8192), ks.view(np.uint8).reshape(5, 256)], 1)
    bt = np.tile(np.arange(5, dtype=np.int32), (R, 1))
    lp, mp, _ = O.mqa_logits_paged(q.view(torch.uint8).numpy(), pages, w, end, bt, N, 1)
    assert np.array_equal(mr, mp)
    both = O.mask_bits(mr, N)
    assert np.array_equal(lr[both], lp[both])


def test_kstore_oracle_equals_workload_quantisation():
    """The writer's restatement produces the same pages as the workloads' per-token amax/448
    quantisation + packing (the K every config's cache is built from), through a scattered slot map."""
    from hcu_ops.workloads import pack_index_k_pages, quant_rows_fp8

    g = torch.Generator().manual_seed(3)
    n_pages = 6
    k = torch.randn(n_pages * 64, 128, generator=g) * 3.0
    k[5] = 0.0                       # amax 0 -> clamped scale
    k[6, 17] = 1e30                  # one huge value, the rest flush to 0 in fp8
    kf, ks = quant_rows_fp8(k)
    ref = pack_index_k_pages(kf, ks).view(n_pages, -1).numpy()
    perm = torch.randperm(n_pages * 64, generator=g)
    loc = perm.to(torch.int32).numpy()
    # token i of k_perm goes to slot loc[i] = perm[i]; so k_perm[i] = k[perm[i]]
    got = O.quant_store_index_k(k[perm].numpy(), loc, np.zeros((n_pages, 64 * 132), np.uint8))
    assert np.array_equal(got, ref)
    # out-of-range slots are skipped
    bad = O.quant_store_index_k(k[:2].numpy(), np.array([-1, n_pages * 64], np.int32), np.zeros((n_pages, 64 * 132), np.uint8))
    assert not bad.any()


def test_mla_writer_restatement_round_trips_through_the_dequant():
    """The MLA writer's restatement (oracle/mla.py) and the 656-byte dequant's restatement agree on
    the slot layout: fp8 bytes times group scales give back the normed latent within fp8 precision,
    and the rope part is the rotated k_pe bit for bit; a rotation keeps the pairs' norms."""
    from oracle import mla as M

    g = torch.Generator().manual_seed(3)
    T, slots = 6, 16
    kv_c = M.to_bf(torch.randn(T, 512, generator=g).numpy() * 3)
    w = M.to_bf((torch.rand(512, generator=g) * 2).numpy())
    k_pe = M.to_bf(torch.randn(T, 64, generator=g).numpy())
    q_pe = M.to_bf(torch.randn(T, 4, 64, generator=g).numpy())
    ang = torch.arange(100)[:, None] * (10000.0 ** (-torch.arange(32) / 32))
    cache = M.to_bf(torch.cat([ang.cos(), ang.sin()], dim=-1).numpy())
    pos = np.array([0, 5, 99, 17, 42, 3])
    loc = np.array([15, 0, 7, 3, 9, 11])
    for neox in (False, True):
        q_out, y, kp, buf = M.rope_qout_kv_store(pos, q_pe, kv_c, w, 1e-6, k_pe, cache, neox,
                                                 np.zeros((slots, 656), np.uint8), loc)
        deq = O.dequant_mla_656(buf.reshape(slots, 1, 656), loc.astype(np.int32))  # bf16 bits [T, 1, 576]
        yf = M.bf(y)
        dv = M.bf(deq.reshape(T, 576)[:, :512])
        scale = np.abs(yf).reshape(T, 4, 128).max(axis=2) / 448
        assert (np.abs(dv - yf) <= 2.0 ** -4 * np.abs(yf) + np.repeat(scale, 128, axis=1) * 2.0 ** -9).all()
        assert np.array_equal(deq.reshape(T, 576)[:, 512:], kp)
        assert np.array_equal(q_out[0], q_pe[0])  # position 0: cos 1, sin 0
        r = np.arange(32)
        xi, yi = (r, 32 + r) if neox else (2 * r, 2 * r + 1)
        n0 = M.bf(k_pe[:, xi]) ** 2 + M.bf(k_pe[:, yi]) ** 2
        n1 = M.bf(kp[:, xi]) ** 2 + M.bf(kp[:, yi]) ** 2
        assert np.allclose(n0, n1, rtol=2 ** -5, atol=1e-3)
