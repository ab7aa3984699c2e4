"""Context-parallel (KV-range) prefill indexer over torch.distributed.

Rank r of P owns the contiguous KV range ``[r*N/P, (r+1)*N/P)``.  For every
query row it scores only that range (ragged logits kernel), selects a local
top-2048 of (uint32 key, global token index) in ascending token order, and the
ranks exchange and merge those lists:

* ``mode="rowshard"`` (default): an all-to-all hands rank r the P lists of its
  1/P share of the rows, rank r merges them, and an all-gather of the final
  int32 indices gives every rank the whole ``[rows, 2048]`` result.  Each rank
  receives ``(P-1)/P`` of one rank's lists instead of ``P-1`` whole lists.
* ``mode="allgather"``: every rank all-gathers all lists and merges all rows.

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


def kv_range(rank: int, world: int, n_tokens: int):
    """Contiguous KV range of a rank; boundaries are multiples of 16 (mask words stay aligned)."""
    def b(r):
        return (n_tokens * r // world) // 16 * 16 if r < world else n_tokens

    return b(rank), b(rank + 1)


def local_rows(row_end: torch.Tensor, lo: int, hi: int) -> torch.Tensor:
    """Visible length of each row inside [lo, hi) for causal rows that see [0, row_end)."""
    return (row_end.clamp(max=hi) - lo).clamp(min=0).to(torch.int32)


def cp_prefill_topk(q, k_fp8_local, k_scale_local, weights, row_end, n_tokens, group=None, mode="rowshard",
                    ops=None):
    """Global top-2048 token indices of every query row, computed over P KV ranges.

    q: fp8 ``[rows, H, 128]`` (replicated); ``k_fp8_local``/``k_scale_local``: this rank's
    KV range ``kv_range(rank, P, n_tokens)``; ``row_end``: int32 ``[rows]`` global visible end
    (row r sees tokens ``[0, row_end[r])``).  Returns int32 ``[rows, 2048]`` (-1 pads) on
    every rank.  Every rank takes the same collective steps in the same order.
    """
    ops = ops or CudaOps()
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    rows = q.shape[0]
    dev = q.device
    lo, hi = kv_range(rank, world, n_tokens)
    assert k_fp8_local.shape[0] == hi - lo, "local K does not match this rank's range"
    lens = local_rows(row_end, lo, hi)
    zeros = torch.zeros_like(lens)
    lg, mk = ops.logits(q, k_fp8_local, k_scale_local, weights, zeros, lens)
    width = hi - lo
    gtab = (torch.arange(width, dtype=torch.int32, device=dev) + lo).expand(rows, width)
    if world == 1:  # one range: the canonical top-k is the answer (no exchange, no merge)
        return ops.topk(lg, mk, lens, gtab)
    idx, keys = ops.local_topk(lg, mk, lens, gtab)
    vis = row_end.clamp(max=n_tokens).to(torch.int32)
    if mode == "allgather":
        all_k = torch.empty((world * rows, TOPK), dtype=keys.dtype, device=dev)
        all_i = torch.empty((world * rows, TOPK), dtype=idx.dtype, device=dev)
        dist.all_gather_into_tensor(all_k, keys.contiguous(), group=group)
        dist.all_gather_into_tensor(all_i, idx.contiguous(), group=group)
        return ops.merge(all_k.view(world, rows, TOPK), all_i.view(world, rows, TOPK), vis)
    # row-sharded exchange: rank d merges rows [d*rps, (d+1)*rps)
    rps = (rows + world - 1) // world
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
