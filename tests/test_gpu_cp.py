"""GPU parity of the context-parallel merge on one device: P per-range local top-k lists
merged by cp_topk_merge equal the single-range top-k exactly (set and order)."""
import numpy as np
import pytest
import torch

from indexer_testlib import make_scores
from oracle import indexer as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("parts", [1, 2, 4, 8])
@pytest.mark.parametrize("dist", ["relu_sum", "ties", "sparse2", "const", "narrow"])
def test_cp_merge_equals_single_range(hcu, dev, parts, dist):
    rows, N = 12, 24576
    x, mask, _, _ = make_scores(rows, N, dist, W=N, seed=parts)
    vis = torch.tensor([N, 3000, 2048, 100, 6001, 2049, 1, 12000, 20000, 4097, 8191, 0], dtype=torch.int32)
    ident = torch.arange(N, dtype=torch.int32).repeat(rows, 1)
    full = O.topk_transform(x.numpy(), mask.numpy(), vis.numpy(), ident.numpy())

    xd, md = x.to(dev), mask.to(dev)
    bounds = np.linspace(0, N, parts + 1).astype(int)
    keys = torch.zeros(parts, rows, 2048, dtype=torch.int32, device=dev)
    gidx = torch.full((parts, rows, 2048), -1, dtype=torch.int32, device=dev)
    for p in range(parts):
        a, b = int(bounds[p]), int(bounds[p + 1])
        local_len = (torch.clamp(vis, max=b) - a).clamp(min=0).to(torch.int32).to(dev)
        # local score view of the range (mask words stay aligned when a % 16 == 0)
        assert a % 16 == 0
        sx = xd[:, a:b].contiguous()
        sm = md[:, a // 16: (b + 15) // 16].contiguous()
        pt = (torch.arange(b - a, dtype=torch.int32, device=dev) + a).repeat(rows, 1)
        idx, k = hcu.topk_keys(sx, sm, local_len, pt)
        keys[p], gidx[p] = k, idx
    merged = hcu.cp_topk_merge(keys, gidx, vis.to(dev))
    assert np.array_equal(merged.cpu().numpy(), full)


def _ranges(N, parts):
    b = [(N * p // parts) // 16 * 16 for p in range(parts)] + [N]
    return [(b[p], b[p + 1]) for p in range(parts)]


def _local(xd, md, vis, a, b, dev):
    rows = xd.shape[0]
    lens = (torch.clamp(vis, max=b) - a).clamp(min=0).to(torch.int32).to(dev)
    sx = xd[:, a:b].contiguous()
    sm = md[:, a // 16: (b + 15) // 16].contiguous()
    pt = (torch.arange(b - a, dtype=torch.int32, device=dev) + a).expand(rows, b - a)
    return sx, sm, lens, pt


def test_cp_bound_matches_oracle(hcu, dev):
    """The sampled bound is bit-exact against its restatement: long and short rows, an empty
    local range, a range smaller than the sample count, one where every token passes, and a range
    too small to constrain the bound."""
    rows, W = 10, 20000
    x, mask, _, _ = make_scores(rows, W, "relu_sum", W=W, seed=31)
    lens = torch.tensor([20000, 20000, 0, 1500, 300, 20000, 5000, 2049, 20000, 40], dtype=torch.int32)
    totals = torch.tensor([160000, 20000, 50000, 1500, 2100, 2048, 9000, 100000, 40000, 100000], dtype=torch.int32)
    ref = O.cp_local_bound(x.numpy(), mask.numpy(), lens.numpy(), totals.numpy())
    got = hcu.cp_local_bound(x.to(dev), mask.to(dev), lens.to(dev), totals.to(dev)).cpu().numpy()
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("cap", [1024, 2048])
def test_cp_filter_matches_oracle(hcu, dev, cap):
    rows, W = 10, 16384
    x, mask, lens, _ = make_scores(rows, W, "ties", W=W, ragged=True, seed=cap)
    pt = (torch.arange(W, dtype=torch.int32) + 5000).expand(rows, W)
    totals = torch.full((rows,), 130000, dtype=torch.int32)
    bounds = torch.from_numpy(O.cp_local_bound(x.numpy(), mask.numpy(), lens.numpy(), totals.numpy()))
    bounds[3] = -2**31  # key 0: every token passes (past the candidate capacity: the flag)
    kr = np.sort(np.where(O.mask_bits(mask.numpy(), W)[5, :int(lens[5])], O.to_key(x.numpy()[5, :int(lens[5])]),
                          O.ZERO_KEY).astype(np.uint32))[::-1]
    bounds[5] = int(np.int64(kr[3000]) - 2**31)  # ~3000 candidates: more than the slots, within capacity
    k, g, cnt, f = O.cp_filter(x.numpy(), mask.numpy(), lens.numpy(), pt.numpy(), bounds.numpy(), cap)
    rps, P = 4, 3  # the rows land row-sharded in a [P, 2, rps, cap] exchange buffer
    send = torch.full((P, 2, rps, cap), 7, dtype=torch.int32, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    hcu.cp_filter(x.to(dev), mask.to(dev), lens.to(dev), pt.to(dev), bounds.to(dev), send, flag)
    s = send.cpu().numpy()
    for r in range(rows):
        assert np.array_equal(s[r // rps, 0, r % rps].view(np.uint32), k[r]), r
        assert np.array_equal(s[r // rps, 1, r % rps], g[r]), r
    assert int(flag.item()) == f == 1


def _bounded_on_one_gpu(hcu, dev, x, mask, vis, parts, cap):
    """P ranges on one device through the bounded protocol (bounds -> MIN -> filter into row-sharded
    buffers -> exchange by indexing -> merge); returns (result rows, flag)."""
    rows, N = x.shape
    xd, md, visd = x.to(dev), mask.to(dev), vis.to(dev)
    rps = (rows + parts - 1) // parts
    pad = rps * parts - rows
    rng = _ranges(N, parts)
    locs = [_local(xd, md, vis, a, b, dev) for a, b in rng]
    bounds = torch.stack([hcu.cp_local_bound(sx, sm, lens, visd) for sx, sm, lens, _ in locs]).min(0).values
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    sends = []
    for sx, sm, lens, pt in locs:
        send = torch.empty((parts, 2, rps, cap), dtype=torch.int32, device=dev)
        if pad:
            send[parts - 1, 1, rps - pad:] = -1
        hcu.cp_filter(sx, sm, lens, pt, bounds, send, flag)
        sends.append(send)
    vis_p = torch.cat([visd, torch.zeros(pad, dtype=torch.int32, device=dev)])
    outs = []
    for d in range(parts):
        recv = torch.stack([sends[src][d] for src in range(parts)]).contiguous()
        outs.append(hcu.cp_topk_merge_lists(recv, vis_p[d * rps:(d + 1) * rps].contiguous(), flag))
    return torch.cat(outs)[:rows].cpu().numpy(), int(flag.item())


@pytest.mark.parametrize("parts", [2, 4, 8])
@pytest.mark.parametrize("dist", ["relu_sum", "ties", "narrow"])
def test_cp_bounded_exchange_on_one_gpu(hcu, dev, parts, dist):
    """The bounded exchange with 2048-slot lists equals the single-range top-k exactly, also for rows
    that one range holds almost entirely."""
    rows, N = 13, 32768
    x, mask, _, _ = make_scores(rows, N, dist, W=N, seed=parts + 100)
    vis = torch.tensor([N, 30000, 2048, 100, 6001, 2049, 1, 12000, 20000, 4097, 8191, 0, 25000], dtype=torch.int32)
    ident = torch.arange(N, dtype=torch.int32).repeat(rows, 1)
    full = O.topk_transform(x.numpy(), mask.numpy(), vis.numpy(), ident.numpy())
    got, flag = _bounded_on_one_gpu(hcu, dev, x, mask, vis, parts, 2048)
    assert flag == 0
    assert np.array_equal(got, full)


@pytest.mark.parametrize("dist", ["relu_sum", "ties"])
def test_cp_truncated_lists(hcu, dev, dist):
    """1024-slot lists at P = 8 (the default there): long rows spread over the ranges merge exactly
    with no flag; a row that one range holds almost entirely overflows its list, whose marker is not
    below the row's threshold, and the merge raises the flag (the caller's rerun)."""
    rows, N, parts = 12, 65536, 8
    x, mask, _, _ = make_scores(rows, N, dist, W=N, seed=7)
    ident = torch.arange(N, dtype=torch.int32).repeat(rows, 1)
    vis = torch.tensor([N, 60000, 50000, 40000, 65000, 33000, 64000, 58000, 45000, 38000, 62000, 36000],
                       dtype=torch.int32)
    full = O.topk_transform(x.numpy(), mask.numpy(), vis.numpy(), ident.numpy())
    got, flag = _bounded_on_one_gpu(hcu, dev, x, mask, vis, parts, 1024)
    assert flag == 0
    assert np.array_equal(got, full)
    vis[3] = 7000  # range 0 (8192 tokens) holds the whole row: its 1023rd largest key is above the threshold
    _, flag = _bounded_on_one_gpu(hcu, dev, x, mask, vis, parts, 1024)
    assert flag == 1


def test_cp_merge_lists_flags_a_missed_bound(hcu, dev):
    """Lists holding fewer than 2048 entries for a long row raise the flag (not the device status)."""
    rows, cap, P = 3, 1024, 2
    recv = torch.full((P, 2, rows, cap), -1, dtype=torch.int32, device=dev)
    recv[:, 0] = 5
    recv[0, 1, :, :100] = torch.arange(100, dtype=torch.int32, device=dev)
    lengths = torch.tensor([5000, 100, 2048], dtype=torch.int32, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    out = hcu.cp_topk_merge_lists(recv, lengths, flag).cpu().numpy()
    assert int(flag.item()) == 1
    assert hcu.read_device_status(clear=False) == 0
    assert np.array_equal(out[1], np.where(np.arange(2048) < 100, np.arange(2048), -1))
    assert np.array_equal(out[2], np.arange(2048))


def _peer_on_one_gpu(hcu, dev, x, mask, vis, parts, cap, steps=2):
    """The peer-memory exchange with `parts` emulated ranks on one device: every phase is issued for
    all ranks before the next phase (so every wait is already satisfied when its kernel starts).
    Returns (every rank's rows after the last step, redo count of rank 0)."""
    from hcu_ops.cp import PeerExchange

    rows, N = x.shape
    xd, md, visd = x.to(dev), mask.to(dev), vis.to(dev)
    locs = [_local(xd, md, vis, a, b, dev) for a, b in _ranges(N, parts)]
    exs = PeerExchange.emulated(parts, rows, dev, cap)
    for _ in range(steps):
        for ex in exs:
            ex.begin()
        for ex, (sx, sm, lens, _) in zip(exs, locs):
            ex.bound(sx, sm, lens, visd)
        for ex, (sx, sm, lens, pt) in zip(exs, locs):
            ex.filter(sx, sm, lens, pt)
        for ex in exs:
            ex.merge(visd)
        for ex in exs:
            ex.finish()
        for ex, loc in zip(exs, locs):
            ex.redo_lists(*loc)
        for ex in exs:
            ex.merge(visd, exact=True)
        for ex in exs:
            ex.finish(exact=True)
    return [ex.out[:rows].cpu().numpy() for ex in exs], exs[0].reruns()


@pytest.mark.parametrize("parts,cap", [(2, 2048), (4, 2048), (8, 1024)])
@pytest.mark.parametrize("dist", ["relu_sum", "ties"])
def test_cp_peer_exchange_on_one_gpu(hcu, dev, parts, cap, dist):
    """Bounds, lists and merged rows stored into the emulated ranks' buffers with per-step flags:
    every rank ends with the single-range top-k of every row, over two steps (the flags of the second
    step carry the next step number).  With 2048-slot lists no redo is needed; with 1024-slot lists
    (P = 8) row 4 (6001 tokens, ~1400 of its top-2048 in range 0) overflows its list and the step is
    redone exactly on the device."""
    rows, N = 13, 32768
    x, mask, _, _ = make_scores(rows, N, dist, W=N, seed=parts + 200)
    vis = torch.tensor([N, 30000, 2048, 100, 6001, 2049, 1, 12000, 20000, 4097, 8191, 0, 25000], dtype=torch.int32)
    full = O.topk_transform(x.numpy(), mask.numpy(), vis.numpy(), torch.arange(N, dtype=torch.int32).repeat(rows, 1)
                            .numpy())
    outs, reruns = _peer_on_one_gpu(hcu, dev, x, mask, vis, parts, cap)
    assert reruns == (0 if cap == 2048 else 2)
    for r, o in enumerate(outs):
        assert np.array_equal(o, full), r


def test_cp_peer_exchange_exact_redo(hcu, dev):
    """A row that one range holds almost entirely overflows that range's 1024-slot list; its marker
    is not below the row's threshold, the merge flags the step and every rank redoes it with local
    top-2048 lists on the device (no host read): the result is still exact, and the redo counted."""
    rows, N, parts = 12, 65536, 8
    x, mask, _, _ = make_scores(rows, N, "relu_sum", W=N, seed=7)
    vis = torch.tensor([N, 60000, 50000, 7000, 65000, 33000, 64000, 58000, 45000, 38000, 62000, 36000],
                       dtype=torch.int32)
    full = O.topk_transform(x.numpy(), mask.numpy(), vis.numpy(), torch.arange(N, dtype=torch.int32).repeat(rows, 1)
                            .numpy())
    outs, reruns = _peer_on_one_gpu(hcu, dev, x, mask, vis, parts, 1024, steps=2)
    assert reruns == 2
    for r, o in enumerate(outs):
        assert np.array_equal(o, full), r


def test_cp_peer_wait_expires_and_device_stays_usable(hcu, dev, request):
    """Failure detection without a fault: with the wait limit set to 1 ms, a finish kernel waits for
    flags that no rank ever sets.  It gives up, records HCU_STATUS_WAIT_TIMEOUT and flags the step,
    the launch returns, and the next exchange on the same device is exact with a clean status."""
    import time

    from hcu_ops.cp import PeerExchange

    request.node.allowed_status = 1
    exs = PeerExchange.emulated(2, 64, dev, 2048)
    hcu._C.set_wait_limit_ns(1_000_000)
    try:
        exs[0].begin()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        exs[0].finish()  # rank 1 never merges: its flag for this step never arrives
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        st = hcu.read_device_status(clear=True)
    finally:
        hcu._C.set_wait_limit_ns(0)
    assert st == 1, st
    assert int(exs[0].ws[8].item()) == 1
    assert dt < 0.5, dt
    rows, N = 9, 20000
    x, mask, _, _ = make_scores(rows, N, "mixed", W=N, seed=3)
    vis = torch.tensor([N, 15000, 2048, 100, 6001, 2049, 1, 12000, 20000], dtype=torch.int32)
    full = O.topk_transform(x.numpy(), mask.numpy(), vis.numpy(), torch.arange(N, dtype=torch.int32).repeat(rows, 1)
                            .numpy())
    outs, _ = _peer_on_one_gpu(hcu, dev, x, mask, vis, 2, 2048, steps=1)
    for o in outs:
        assert np.array_equal(o, full)
    assert hcu.read_device_status(clear=True) == 0
