"""CPU multi-process test of the context-parallel driver (gloo, world size 2 and 3).

The device ops are replaced by oracle-backed CPU stand-ins so the distributed plumbing (KV-range
split, local selection in token order, row-sharded all-to-all / all-gather exchange, merge) is
exercised without a GPU; the result must equal the single-range top-k exactly."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class OracleOps:
    def logits(self, q, k_fp8, k_scale, weights, rs, re):
        from oracle import indexer as O

        lg, m, _ = O.mqa_logits_ragged(q.view(torch.uint8).numpy(), k_fp8.view(torch.uint8).numpy(),
                                       k_scale.numpy(), weights.numpy(), rs.numpy(), re.numpy())
        return torch.from_numpy(lg), torch.from_numpy(m)

    def local_topk(self, score, mask, lengths, pt):
        from oracle import indexer as O

        idx, keys = O.topk_transform(score.numpy(), mask.numpy(), lengths.numpy(),
                                     np.ascontiguousarray(pt.numpy()), return_keys=True)
        for r in range(idx.shape[0]):  # ascending token order, as the device op emits
            v = idx[r] >= 0
            o = np.argsort(idx[r][v], kind="stable")
            idx[r][v] = idx[r][v][o]
            keys[r][v] = keys[r][v][o]
        return torch.from_numpy(idx), torch.from_numpy(keys.view(np.int32))

    def topk(self, score, mask, lengths, pt):
        from oracle import indexer as O

        return torch.from_numpy(O.topk_transform(score.numpy(), mask.numpy(), lengths.numpy(),
                                                 np.ascontiguousarray(pt.numpy())))

    def merge(self, keys, gidx, lengths):
        from oracle import indexer as O

        return torch.from_numpy(O.cp_merge(keys.numpy().view(np.uint32), gidx.numpy(), lengths.numpy()))

    def bound(self, score, mask, lengths, totals):
        from oracle import indexer as O

        return torch.from_numpy(O.cp_local_bound(score.numpy(), mask.numpy(), lengths.numpy(), totals.numpy()))

    def filter(self, score, mask, lengths, pt, bounds, send, flag):
        from oracle import indexer as O

        P, _, rps, cap = send.shape
        k, g, _, f = O.cp_filter(score.numpy(), mask.numpy(), lengths.numpy(), np.ascontiguousarray(pt.numpy()),
                                 bounds.numpy(), cap)
        for r in range(score.shape[0]):
            send[r // rps, 0, r % rps] = torch.from_numpy(k[r].view(np.int32))
            send[r // rps, 1, r % rps] = torch.from_numpy(g[r])
        flag |= f

    def merge_lists(self, recv, lengths, flag):
        from oracle import indexer as O

        out, f = O.cp_merge_lists(recv[:, 0].numpy().view(np.uint32), recv[:, 1].numpy(), lengths.numpy())
        flag |= f
        return torch.from_numpy(out)


class MissOps(OracleOps):
    """A bound above every key: the lists hold fewer than 2048 entries, the merge flags it."""

    def bound(self, score, mask, lengths, totals):
        return torch.full((score.shape[0],), 2**31 - 1, dtype=torch.int32)


class OverflowOps(OracleOps):
    """A bound of 0: every token passes, the lists overflow, the filter flags it."""

    def bound(self, score, mask, lengths, totals):
        return torch.full((score.shape[0],), -2**31, dtype=torch.int32)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, variant, q):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    for p in (os.path.dirname(here), os.path.join(os.path.dirname(here), "sglang0.5.18-opt_b200"), here):
        sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    if variant == "short_lists":  # 1024-slot lists: truncated lists and their markers
        os.environ["HCU_CP_LIST_LEN"] = "1024"
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from hcu_ops.cp import cp_prefill_topk, kv_range
        from hcu_ops.workloads import make_ragged

        w = make_ragged(23, 2600, heads=32, seed=11)  # same seed on every rank: replicated q
        N = w["k_fp8"].shape[0]
        cr = 23 if variant in ("balanced", "weighted") else 0
        shares = [1.0 + 0.5 * r for r in range(world)] if variant == "weighted" else None  # unequal GPU rates
        lo, hi = kv_range(rank, world, N, causal_rows=cr, shares=shares)
        ops = {"miss": MissOps, "overflow": OverflowOps}.get(variant, OracleOps)()
        out = cp_prefill_topk(w["q"], w["k_fp8"][lo:hi].contiguous(), w["k_scale"][lo:hi].contiguous(),
                              w["weights"], w["row_end"], N, mode=mode, ops=ops, bounded=variant != "exact",
                              causal_rows=cr, shares=shares)
        q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,mode,variant", [(1, "rowshard", "bounded"), (2, "rowshard", "bounded"),
                                                (2, "rowshard", "exact"), (2, "allgather", "exact"),
                                                (3, "rowshard", "bounded"), (2, "rowshard", "miss"),
                                                (3, "rowshard", "overflow"), (3, "rowshard", "balanced"),
                                                (2, "rowshard", "short_lists"), (3, "rowshard", "weighted")])
def test_cp_driver_equals_single_range(world, mode, variant):
    """Every rank's result equals the single-range top-k: the bounded exchange, the exact one,
    and the bounded exchange whose bound misses (too high) or overflows the lists (too low),
    which every rank detects and reruns exactly; and ranges balanced by visible pairs."""
    from hcu_ops.workloads import make_ragged
    from oracle import indexer as O

    w = make_ragged(23, 2600, heads=32, seed=11)
    lg, m, _ = O.mqa_logits_ragged(w["q"].view(torch.uint8).numpy(), w["k_fp8"].view(torch.uint8).numpy(),
                                   w["k_scale"].numpy(), w["weights"].numpy(), w["row_start"].numpy(),
                                   w["row_end"].numpy())
    N = lg.shape[1]
    ident = np.tile(np.arange(N, dtype=np.int32), (23, 1))
    ref = O.topk_transform(lg, m, w["row_end"].numpy(), ident)

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, variant, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, out = q.get(timeout=240)
        got[r] = out
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert np.array_equal(got[r], ref), f"rank {r}"


@pytest.mark.parametrize("value, world, ok", [("1024", 8, True), ("2048", 2, True), ("256", 8, True),
                                              ("512", 2, False), ("1000", 8, False), ("4096", 2, False),
                                              ("128", 16, False), ("x", 8, False)])
def test_cp_list_len_override_is_checked(monkeypatch, value, world, ok):
    """HCU_CP_LIST_LEN is validated on the host before any collective: a power of two in
    [256, 2048] whose product with the world size covers 2048 entries per row."""
    from hcu_ops.cp import list_len

    monkeypatch.setenv("HCU_CP_LIST_LEN", value)
    if ok:
        assert list_len(world) == int(value)
    else:
        with pytest.raises(ValueError):
            list_len(world)


def test_kv_range_shares():
    """Weighted ranges tile [0, N) in order with 16-token boundaries; without causal rows the token
    counts follow the weights, with causal rows the visible pairs do."""
    from hcu_ops.cp import kv_range

    N, R = 131072, 16384
    shares = [1.0, 1.2, 0.9, 1.1, 1.0, 0.8, 1.3, 1.0]
    for cr in (0, R):
        rng = [kv_range(r, 8, N, causal_rows=cr, shares=shares) for r in range(8)]
        assert rng[0][0] == 0 and rng[-1][1] == N
        assert all(rng[i][1] == rng[i + 1][0] for i in range(7))
        assert all(a % 16 == 0 for a, _ in rng)

        def pairs(x):  # visible pairs in [0, x) for rows seeing [0, N - R + i + 1)
            if not cr:
                return x
            p = N - R
            if x <= p:
                return R * x
            d = x - p
            return R * p + d * (d + 1) // 2 + (R - d) * d

        tot = pairs(N)
        for r, (a, b) in enumerate(rng):
            assert abs((pairs(b) - pairs(a)) / tot - shares[r] / sum(shares)) < 2e-3
    assert kv_range(3, 8, N, causal_rows=R) == kv_range(3, 8, N, causal_rows=R, shares=[2.0] * 8)
    with pytest.raises(ValueError):
        kv_range(0, 2, N, shares=[1.0, 0.0])
