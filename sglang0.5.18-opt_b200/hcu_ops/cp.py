"""Context-parallel (KV-range) prefill indexer over torch.distributed.

Rank r of P owns the contiguous KV range ``[r*N/P, (r+1)*N/P)``.  For every
query row it scores only that range (ragged logits kernel), selects a local
top-2048 of (uint32 key, global token index) in ascending token order, and the
ranks exchange and merge those lists:

* ``mode="rowshard"`` (NCCL; the default with stand-in ops): an all-to-all hands rank r the P lists of its
  1/P share of the rows, rank r merges them, and an all-gather of the final
  int32 indices gives every rank the whole ``[rows, 2048]`` result.  Each rank
  receives ``(P-1)/P`` of one rank's lists instead of ``P-1`` whole lists.
  The lists are bounded (``bounded=True``, default): instead of a local
  top-2048, each rank keeps the tokens at or above the row's bound b, the
  minimum over ranks of a sampled estimate of the row's global threshold on
  each range (one all-reduce MIN of an int32 per row), in lists of C entries
  (``list_len``: 2048, or 1024 from 8 ranks on).  A range with more tokens at or
  above b sends its top-2048 among them when C = 2048 (every token of the row's
  global top-2048 in that range is one of them), else its top-(C - 1) and a
  marker carrying the largest key it may have dropped.  The union is exact when
  every row holds at least 2048 entries (then the global threshold is >= b) and
  the row's threshold is above every marker; the merge flags the rows where that
  fails (and the filter a range past its candidate capacity), one all-reduce MAX
  of the flag tells every rank, and the step then reruns with local top-2048
  lists (the exact path).
* ``mode="allgather"``: every rank all-gathers all lists and merges all rows.
* ``mode="peer"`` (default for the CUDA ops): the bounded exchange without NCCL.  Every rank's
  exchange buffers are mapped into every other rank (symmetric memory over NVLink); the bound,
  filter and merge kernels store their results straight into the consuming ranks' buffers and
  publish per-step flags that the consumers wait for (``PeerExchange``; C ABI ``hcu_cp_peer_*``).
  The exact redo is predicated on a device word that every rank computes identically, so a step
  has no host synchronisation.  When symmetric memory cannot be set up the NCCL row-shard exchange
  is used instead.

The global top-2048 under (key desc, global index asc) is a subset of the union
of the local ones, and the merge writes the single-GPU canonical order, so the
result equals the 1-GPU output exactly.  The path has no counterpart in the
reference (its CP8 is sglang's round-robin query split, ``prefill/p_opt.sh:132-133``).

``ops`` defaults to this package's CUDA ops; tests substitute CPU stand-ins to
exercise the distributed plumbing with the gloo backend.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

TOPK = 2048


class CudaOps:
    """The device ops the CP driver needs (the product path)."""

    def bound(self, score, mask, lengths, totals):
        from . import cp_local_bound

        return cp_local_bound(score, mask, lengths, totals)

    def filter(self, score, mask, lengths, page_table, bounds, send, flag):
        from . import cp_filter

        cp_filter(score, mask, lengths, page_table, bounds, send, flag)

    def merge_lists(self, recv, lengths, flag):
        from . import cp_topk_merge_lists

        return cp_topk_merge_lists(recv, lengths, flag, True)

    def logits(self, q, k_fp8, k_scale, weights, row_start, row_end):
        from . import mqa_logits_ragged

        return mqa_logits_ragged(q, k_fp8, k_scale, weights, row_start, row_end)

    def local_topk(self, score, mask, lengths, page_table):
        from . import topk_keys

        return topk_keys(score, mask, lengths, page_table)

    def topk(self, score, mask, lengths, page_table):
        from . import sparse_mask_topk_transform

        rows = score.shape[0]
        cu = torch.arange(rows + 1, dtype=torch.int32, device=score.device)
        return sparse_mask_topk_transform(score, mask, lengths, page_table, cu)

    def merge(self, keys, gidx, lengths):
        from . import cp_topk_merge

        return cp_topk_merge(keys, gidx, lengths)


def kv_range(rank: int, world: int, n_tokens: int, causal_rows: int = 0, shares=None):
    """Contiguous KV range of a rank; boundaries are multiples of 16 (mask words stay aligned).

    ``causal_rows = 0``: equal token counts.  ``causal_rows = R``: the query rows are the last R
    positions of the context (row i sees tokens [0, n_tokens - R + i + 1)), and the boundaries
    give every rank about the same number of visible (row, token) pairs, so the rank that holds
    the causal triangle takes a longer range instead of idling.  ``shares`` (one positive weight
    per rank, e.g. from ``calibrate_shares``): rank r takes a fraction shares[r] / sum(shares) of
    the tokens (of the visible pairs with ``causal_rows``) instead of an equal one.  Every rank
    must pass the same arguments."""
    if rank >= world:
        return n_tokens, n_tokens
    if shares is not None:
        w = [float(x) for x in shares]
        if len(w) != world or min(w) <= 0:
            raise ValueError("shares: one positive weight per rank")
        cum = [0.0]
        for x in w:
            cum.append(cum[-1] + x)
        frac = [c / cum[-1] for c in cum]
    else:
        frac = [r / world for r in range(world + 1)]
    if causal_rows <= 0:
        def b(r):
            return int(n_tokens * frac[r]) // 16 * 16 if r < world else n_tokens
        return b(rank), b(rank + 1)
    R = min(int(causal_rows), n_tokens)
    p = n_tokens - R

    def pairs(x):  # visible pairs in [0, x)
        if x <= p:
            return R * x
        d = x - p
        return R * p + d * (d + 1) // 2 + (R - d) * d

    total = pairs(n_tokens)

    def b(r):
        if r <= 0:
            return 0
        if r >= world:
            return n_tokens
        target = total * r // world if shares is None else int(total * frac[r])
        lo, hi = 0, n_tokens  # smallest x with pairs(x) >= target, then down to a multiple of 16
        while lo < hi:
            mid = (lo + hi) // 2
            if pairs(mid) >= target:
                hi = mid
            else:
                lo = mid + 1
        return lo // 16 * 16

    return b(rank), b(rank + 1)


def calibrate_shares(group=None, device=None, rows=2048, tokens=32768, reps=5):
    """Relative prefill-logits rates of the ranks' GPUs, for ``kv_range(..., shares=...)``.

    GPUs of one box can differ by tens of percent on the same kernel, and a context-parallel step
    waits for its slowest rank; weighting each rank's range by its measured rate evens out the
    ranks' step times.  Every rank times the ragged logits kernel on the same seeded block (median
    of ``reps`` runs), the times are all-gathered, and each rank gets weight 1 / time (identical
    list on every rank).  A collective step: call it on every rank, once, outside any timed region."""
    from . import mqa_logits_ragged
    from .workloads import make_ragged

    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    w = make_ragged(rows, tokens - rows, heads=64, seed=123, device=dev)
    zeros = torch.zeros_like(w["row_end"])
    for _ in range(2):
        mqa_logits_ragged(w["q"], w["k_fp8"], w["k_scale"], w["weights"], zeros, w["row_end"])
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        mqa_logits_ragged(w["q"], w["k_fp8"], w["k_scale"], w["weights"], zeros, w["row_end"])
        b.record()
        torch.cuda.synchronize(dev)
        times.append(a.elapsed_time(b))
    t = torch.tensor([sorted(times)[len(times) // 2]], dtype=torch.float64, device=dev)
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world > 1:
        allt = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allt, t, group=group)
        ts = [float(x.item()) for x in allt]
    else:
        ts = [float(t.item())]
    return [1.0 / x for x in ts]


def local_rows(row_end: torch.Tensor, lo: int, hi: int) -> torch.Tensor:
    """Visible length of each row inside [lo, hi) for causal rows that see [0, row_end)."""
    return (row_end.clamp(max=hi) - lo).clamp(min=0).to(torch.int32)


def list_len(world: int) -> int:
    """Slots per (rank, row) list of the bounded exchange: 2048 below 8 ranks, 1024 from 8 on
    (HCU_CP_LIST_LEN overrides: a power of two in [256, 2048], times world >= 2048).  A shorter
    list that overflows is truncated to its top entries plus a marker holding the largest key it
    may have dropped; the merge checks the row's threshold against it (a rerun when not above)."""
    import os

    env = os.environ.get("HCU_CP_LIST_LEN")
    if not env:
        return 1024 if world >= 8 else 2048
    try:
        n = int(env)
    except ValueError:
        n = -1
    # checked here, before the step's first collective, so every rank fails at the same point
    if n < 256 or n > TOPK or n & (n - 1) or n * world < TOPK:
        raise ValueError(f"HCU_CP_LIST_LEN={env!r}: need a power of two in [256, {TOPK}] "
                         f"with value x world ({world}) >= {TOPK}")
    return n


# --------------------------------------------------------------------------- peer-memory exchange
_MAX_PARTS = 16  # HCU_CP_MAX_PARTS
_WS_FLAG, _WS_RERUNS, _WS_WORDS = 8, 9, 16


def _peer_layout(parts, rows, rps):
    """int32 offsets of one rank's regions in its exchange allocation (256-byte aligned):
    bounds [P, R] | lists [P, 2, rps, 2048] (also the redo's lists) | out [P * rps, 2048] | sig [5, P]."""
    offs, n = {}, 0
    for name, size in (("bounds", parts * rows), ("lists", parts * 2 * rps * TOPK), ("out", parts * rps * TOPK),
                       ("sig", 5 * parts)):
        offs[name] = n
        n += (size + 63) // 64 * 64
    return offs, n


class PeerExchange:
    """The exchange buffers of one rank and the kernels of one step (``hcu_cp_peer_*``).

    ``bases``: the device address of every rank's exchange allocation as mapped in this process;
    ``local``: this rank's allocation (int32 tensor); ``ws``: this rank's 16-word workspace.  Use
    ``over_group`` (one rank per process, symmetric memory) or ``emulated`` (all ranks in one process
    on one device, for tests: each phase must then be issued for every rank before the next phase).
    The returned rows are a view of the exchange buffer, valid until the next step's merge."""

    def __init__(self, parts, rank, rows, cap, bases, local, ws):
        from . import _C

        self._C = _C
        self.parts, self.rank, self.rows, self.cap = parts, rank, rows, cap
        self.rps = (rows + parts - 1) // parts
        offs, _ = _peer_layout(parts, rows, self.rps)
        self.local, self.ws = local, ws
        self.epoch = 0
        t = torch.zeros(7 + 5 * _MAX_PARTS, dtype=torch.int64)
        t[0], t[1], t[2], t[3], t[4] = parts, rank, rows, self.rps, cap
        t[6] = ws.data_ptr()
        for i, name in enumerate(("bounds", "lists", "lists", "out", "sig")):
            for p in range(parts):
                t[7 + i * _MAX_PARTS + p] = bases[p] + 4 * offs[name]
        self.peers = t
        o = offs["out"]
        self.out = local[o:o + parts * self.rps * TOPK].view(parts * self.rps, TOPK)

    @staticmethod
    def _zeroed(n, dev, alloc):
        t = alloc(n)
        t.zero_()
        return t

    @classmethod
    def over_group(cls, group, rows, dev, cap):
        import os

        # The kernels use plain peer loads and stores only: keep the allocation off NVLink multicast
        # objects (no multimem here, and a rank leaving while bound to one disturbs the others).
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm

        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        rps = (rows + world - 1) // world
        _, n = _peer_layout(world, rows, rps)
        local = symm.empty(n, dtype=torch.int32, device=dev)
        local.zero_()
        pg = group if group is not None else dist.group.WORLD
        hdl = symm.rendezvous(local, pg)
        bases = [hdl.get_remote_tensor(p, (n,), torch.int32).data_ptr() for p in range(world)]
        bases[rank] = local.data_ptr()
        ws = torch.zeros(_WS_WORDS, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group)  # every rank's buffers are zero before any rank's first flag
        ex = cls(world, rank, rows, cap, bases, local, ws)
        ex._hdl = hdl
        return ex

    @classmethod
    def emulated(cls, parts, rows, dev, cap):
        rps = (rows + parts - 1) // parts
        _, n = _peer_layout(parts, rows, rps)
        locals_ = [torch.zeros(n, dtype=torch.int32, device=dev) for _ in range(parts)]
        bases = [t.data_ptr() for t in locals_]
        return [cls(parts, r, rows, cap, bases, locals_[r], torch.zeros(_WS_WORDS, dtype=torch.int32, device=dev))
                for r in range(parts)]

    # ---- the phases of a step, in order
    def begin(self):
        self.epoch += 1
        self.peers[5] = self.epoch

    def bound(self, lg, mk, lens, vis):
        self._C.cp_peer_bound(lg, mk, lens, vis, self.peers)

    def filter(self, lg, mk, lens, gtab):
        self._C.cp_peer_filter(lg, mk, lens, gtab, self.peers)

    def mine(self, vis):
        """This rank's rows' visible totals (rps entries, 0 past the batch)."""
        m = vis[self.rank * self.rps:(self.rank + 1) * self.rps]
        if m.numel() < self.rps:
            m = torch.cat([m, torch.zeros(self.rps - m.numel(), dtype=vis.dtype, device=vis.device)])
        return m.contiguous()

    def merge(self, vis, exact=False):
        self._C.cp_peer_merge(self.mine(vis), exact, self.peers)

    def finish(self, exact=False):
        self._C.cp_peer_finish(exact, self.peers)

    def redo_lists(self, lg, mk, lens, gtab):
        idx, keys = self._C.topk_keys_if(lg, mk, lens, gtab, self.ws[_WS_FLAG:_WS_FLAG + 1])
        self._C.cp_peer_scatter_exact(keys, idx, self.peers)

    def step(self, lg, mk, lens, gtab, vis):
        """One whole step for this rank (one rank per process)."""
        self.begin()
        self.bound(lg, mk, lens, vis)
        self.filter(lg, mk, lens, gtab)
        self.merge(vis)
        self.finish()
        self.redo_lists(lg, mk, lens, gtab)  # the exact redo: does nothing unless the step was flagged
        self.merge(vis, exact=True)
        self.finish(exact=True)
        return self.out[:self.rows]

    def reruns(self):
        """Exact redos so far (reads a device word: synchronises)."""
        return int(self.ws[_WS_RERUNS].item())


_PEER_CACHE = {}


def _peer_exchange(group, rows, dev, world):
    """The cached PeerExchange of (group, rows, device), or None when symmetric memory is unavailable
    (decided identically on every rank: a MIN all-reduce of each rank's setup outcome)."""
    key = (id(group), rows, str(dev), world, list_len(world))
    if key in _PEER_CACHE:
        return _PEER_CACHE[key]
    ex, err = None, ""
    try:
        ex = PeerExchange.over_group(group, rows, dev, list_len(world))
    except Exception as e:  # noqa: BLE001  (no symmetric memory on this system: the NCCL exchange is used)
        err = f"{type(e).__name__}: {e}"
    ok = torch.tensor([1 if ex is not None else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
    if int(ok.item()) == 0:
        ex = None
    _PEER_CACHE[key] = ex
    if ex is None:
        _PEER_CACHE[("error",) + key] = err
    return ex


def cp_prefill_topk(q, k_fp8_local, k_scale_local, weights, row_end, n_tokens, group=None, mode=None,
                    ops=None, bounded=True, causal_rows=0, stats=None, shares=None):
    """Global top-2048 token indices of every query row, computed over P KV ranges.

    q: fp8 ``[rows, H, 128]`` (replicated); ``k_fp8_local``/``k_scale_local``: this rank's
    KV range ``kv_range(rank, P, n_tokens, causal_rows, shares)``; ``row_end``: int32 ``[rows]`` global visible end
    (row r sees tokens ``[0, row_end[r])``).  Returns int32 ``[rows, 2048]`` (-1 pads) on
    every rank.  Every rank takes the same collective steps in the same order.  ``stats`` (optional
    dict): "reruns" is incremented when the bounded exchange had to be redone exactly, "exchange"
    names the exchange used.
    """
    stats = {} if stats is None else stats
    if mode is None:
        mode = "peer" if ops is None else "rowshard"
    ops = ops or CudaOps()
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    rows = q.shape[0]
    dev = q.device
    lo, hi = kv_range(rank, world, n_tokens, causal_rows, shares)
    assert k_fp8_local.shape[0] == hi - lo, "local K does not match this rank's range"
    lens = local_rows(row_end, lo, hi)
    zeros = torch.zeros_like(lens)
    lg, mk = ops.logits(q, k_fp8_local, k_scale_local, weights, zeros, lens)
    width = hi - lo
    gtab = (torch.arange(width, dtype=torch.int32, device=dev) + lo).expand(rows, width)
    if world == 1:  # one range: the canonical top-k is the answer (no exchange, no merge)
        stats["exchange"] = "none (one range)"
        return ops.topk(lg, mk, lens, gtab)
    vis = row_end.clamp(max=n_tokens).to(torch.int32)
    rps = (rows + world - 1) // world  # row-sharded exchange: rank d merges rows [d*rps, (d+1)*rps)
    if mode == "peer":
        ex = _peer_exchange(group, rows, dev, world)
        if ex is not None:
            stats["exchange"] = ("peer memory: bounds, bounded lists and merged rows stored by the kernels into "
                                 "the consuming ranks' buffers over NVLink; exact redo predicated on the device")
            stats["peer_exchange"] = ex
            return ex.step(lg, mk, lens, gtab, vis)
        stats["peer_unavailable"] = _PEER_CACHE.get(("error", id(group), rows, str(dev), world, list_len(world)), "")
        mode = "rowshard"
    if mode == "rowshard" and bounded:
        out = _bounded_rowshard(ops, lg, mk, lens, gtab, vis, rows, rps, world, rank, group)
        if out is not None:
            stats["exchange"] = "nccl: bounded row-sharded lists (all_to_all) + all_gather of merged rows"
            return out[:rows]
        stats["reruns"] = stats.get("reruns", 0) + 1
    stats["exchange"] = f"nccl: exact local top-2048 lists ({mode})"
    idx, keys = ops.local_topk(lg, mk, lens, gtab)
    if mode == "allgather":
        all_k = torch.empty((world * rows, TOPK), dtype=keys.dtype, device=dev)
        all_i = torch.empty((world * rows, TOPK), dtype=idx.dtype, device=dev)
        dist.all_gather_into_tensor(all_k, keys.contiguous(), group=group)
        dist.all_gather_into_tensor(all_i, idx.contiguous(), group=group)
        return ops.merge(all_k.view(world, rows, TOPK), all_i.view(world, rows, TOPK), vis)
    pad = rps * world - rows
    if pad:
        keys = torch.cat([keys, torch.zeros((pad, TOPK), dtype=keys.dtype, device=dev)])
        idx = torch.cat([idx, torch.full((pad, TOPK), -1, dtype=idx.dtype, device=dev)])
        vis = torch.cat([vis, torch.zeros(pad, dtype=vis.dtype, device=dev)])
    send = torch.stack([keys, idx]).view(2, world, rps, TOPK).transpose(0, 1).contiguous()  # [dest, 2, rps, K]
    recv = torch.empty_like(send)  # [src, 2, rps, K]
    dist.all_to_all_single(recv, send, group=group)
    mine = ops.merge(recv[:, 0].contiguous(), recv[:, 1].contiguous(), vis[rank * rps:(rank + 1) * rps].contiguous())
    out = torch.empty((world * rps, TOPK), dtype=mine.dtype, device=dev)
    dist.all_gather_into_tensor(out, mine.contiguous(), group=group)
    return out[:rows]


def _bounded_rowshard(ops, lg, mk, lens, gtab, vis, rows, rps, world, rank, group):
    """The bounded exchange; None when some row's union was not exact (every rank sees the same flag)."""
    dev = lg.device
    cap = list_len(world)
    bounds = ops.bound(lg, mk, lens, vis)
    dist.all_reduce(bounds, op=dist.ReduceOp.MIN, group=group)
    send = torch.empty((world, 2, rps, cap), dtype=torch.int32, device=dev)
    pad = rps * world - rows
    if pad:
        send[world - 1, 1, rps - pad:] = -1  # rows past the batch: empty lists
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.filter(lg, mk, lens, gtab, bounds, send, flag)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    vis_p = torch.cat([vis, torch.zeros(pad, dtype=vis.dtype, device=dev)]) if pad else vis
    mine = ops.merge_lists(recv, vis_p[rank * rps:(rank + 1) * rps].contiguous(), flag)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
    # the gather goes out before the flag is read (one host wait per step, after the last
    # collective); every rank reads the same flag, so all discard it and rerun together
    out = torch.empty((world * rps, TOPK), dtype=mine.dtype, device=dev)
    dist.all_gather_into_tensor(out, mine.contiguous(), group=group)
    if int(flag.item()):
        return None
    return out
