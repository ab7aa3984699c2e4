#!/usr/bin/env python
"""Benchmark of the DSA lightning-indexer path on B200.

Default workload (the decode indexer the metric is quoted on):
64 requests x next_n=2 rows, contexts U[4096, 65536], 64 index heads x 128 dim fp8,
shared shuffled pool of 64-token pages.  One step = one CUDA-graph replay of the
sglang decode call pair: hcu_ops.mqa_logits (tcgen05 fp8 paged logits + mask) ->
hcu_ops.sparse_mask_topk_transform (exact top-2048 + page-table transform).

metric: G-scores/s = (sum over rows of visible KV tokens) / step time.
Multi-GPU (torchrun): the decode indexer does not shard, so every rank runs its
own replica of the workload ("scaling": "weak"); value = all ranks' scores / the
slowest rank's time.  --impl reference times the CPU restatement of the same
pipeline (the reference's kernels are HIP-only) on the host cores, rank 0 only.

Other workloads (--workload): prefill (config 2), dequant (config 3), mla_dequant.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(REPO, "sglang0.5.18-opt_b200")
for _p in (REPO, PKG_ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

L2_BYTES = 126 * 1024 * 1024


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, 1590.0, "fallback"


def _profile_traffic(name):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of a kernel from the
    committed ncu summary profiles/<name>.md (its `dram_bytes_per_launch` row), or None."""
    import re

    path = os.path.join(REPO, "profiles", name + ".md")
    try:
        m = re.search(r"dram_bytes_per_launch\s*\|\s*(\d+)", open(path).read())
        return int(m.group(1)) if m else None
    except Exception:  # noqa: BLE001
        return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][2]),
                "reasons": reasons, "samples": len(rows)}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------------------------------------
# decode (config 1) -- the headline
# ------------------------------------------------------------------------------------------------
def decode_inputs(device, seed):
    from hcu_ops.workloads import config1

    return config1(device=device, seed=seed)


def decode_alg_bytes(w):
    """Algorithmic HBM bytes of one logits launch: each group's K pages read once (128 fp8 + 4 B
    scale per token), q + weights, block-table entries, logits written at every visible token,
    and the mask words of the full width (each processed tile's words, the rest zeroed by the kernel)."""
    import torch

    lens = w["context_lens"].long().cpu()
    G, H = w["group_size"], w["heads"]
    B = lens.numel()
    glen = lens.view(-1, G).max(1).values
    k_bytes = int((glen * 132).sum())
    bt_bytes = int(((glen + 63) // 64).sum() * 4)
    q_bytes = B * H * 128 + B * H * 4
    logits_bytes = int(lens.sum() * 4)
    mask_bytes = B * (w["max_context_len"] // 16) * 2 + int(((glen + 127) // 128).sum() * G * 16)
    del torch
    return k_bytes + bt_bytes + q_bytes + logits_bytes + mask_bytes


def run_decode(args, world, rank, local):
    import torch

    import hcu_ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = decode_inputs(dev, seed=rank)
    pairs = int(w["context_lens"].long().sum())
    lens, pt, cu = w["context_lens"], w["page_table_size_1"], w["cu_seqlens_q"]

    def step():
        lg, mk = hcu_ops.mqa_logits(w["q"], w["kv_cache"], w["weights"], lens, w["block_table"],
                                    w["max_context_len"], w["group_size"], hist_lens=lens)
        return hcu_ops.sparse_mask_topk_transform(lg, mk, lens, pt, cu, 2048)

    def logits_only():
        return hcu_ops._C.mqa_logits_hist(w["q"], w["kv_cache"], w["weights"], lens, w["block_table"],
                                          w["max_context_len"], w["group_size"], 0, 0, None)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(max(args.warmup, 3)):
            step()
            logits_only()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = step()
    g_lg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_lg):
        logits_only()
    for _ in range(max(args.warmup, 3)):
        g.replay()
        g_lg.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    # ---- headline: K graph replays of the pipeline (inputs resident in HBM; K pool > L2)
    with ClockSampler(local) as clk:
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            g.replay()
        e1.record(stream)
        barrier()
    ms = e0.elapsed_time(e1) / args.steps
    # ---- dominant kernel alone (the logits op) for the roofline
    barrier()
    l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0.record(stream)
    for _ in range(args.steps):
        g_lg.replay()
    l1.record(stream)
    barrier()
    ms_logits = l0.elapsed_time(l1) / args.steps
    # ---- e2e through the public API with host buffers: every step copies that step's inputs (query rows,
    # head weights, context lengths, block table) from pinned host memory and reads the result back.  The KV
    # cache and the per-token page table (page_table_size_1, built on the device from the request-to-token
    # pool by the serving engine's metadata step) are device state, like the cache itself.
    host = {k: w[k].cpu().pin_memory() for k in ("q", "weights", "context_lens", "block_table")}
    dev_in = {k: torch.empty_like(w[k]) for k in host}
    res_host = torch.empty((lens.numel(), 2048), dtype=torch.int32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = res_host.numel() * 4

    def e2e_step():
        for k, t in host.items():
            dev_in[k].copy_(t, non_blocking=True)
        lg, mk = hcu_ops.mqa_logits(dev_in["q"], w["kv_cache"], dev_in["weights"], dev_in["context_lens"],
                                    dev_in["block_table"], w["max_context_len"], w["group_size"],
                                    hist_lens=dev_in["context_lens"])
        o = hcu_ops.sparse_mask_topk_transform(lg, mk, dev_in["context_lens"], w["page_table_size_1"], cu, 2048)
        res_host.copy_(o, non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier()
    e2e_steps = min(args.steps, 200)
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    x1.record(stream)
    barrier()
    ms_e2e = x0.elapsed_time(x1) / e2e_steps
    st = hcu_ops.read_device_status(clear=True)
    ok = torch.equal(res_host, out.cpu())

    t = torch.tensor([ms, ms_logits, ms_e2e, float(pairs)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = t.clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        sm_ = t.clone()
        torch.distributed.all_reduce(sm_, op=torch.distributed.ReduceOp.SUM)
        ms, ms_logits, ms_e2e = mx[0].item(), mx[1].item(), mx[2].item()
        total_pairs = sm_[3].item()
    else:
        total_pairs = float(pairs)
    if rank != 0:
        return None
    hbm, _, src = _peaks()
    alg = decode_alg_bytes(w)
    achieved = alg / (ms_logits * 1e-3) / 1e9
    traffic = _profile_traffic("mqa_logits_paged_config1")
    rec = {
        "metric": "indexer G-scores/s (rows x visible KV tokens / s), decode logits + top-2048",
        "value": total_pairs / (ms * 1e-3) / 1e9,
        "unit": "G-scores/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8e4m3 x fp8e4m3 -> fp32",
        "data": "synthetic (seeded; q,K ~ N(0,1) per-row/per-token amax/448 fp8; w ~ N(0,1)/8)",
        "config": {"workload": "config1: decode 64 req x next_n 2 (128 rows), ctx U[4096,65536], "
                               "64 heads x 128, 64-token pages, shuffled pool; CUDA-graph replay",
                   "rows": int(lens.numel()), "heads": w["heads"], "width": w["max_context_len"],
                   "pairs_per_gpu": pairs, "kv_pool_bytes": int(w["kv_cache"].numel()),
                   "l2": "no flush: K pool > 126 MB L2", "parallelism": f"replicas x{world}"},
        "top_k_rows_per_s": lens.numel() * world / (ms * 1e-3),
        "logits_op_ms": ms_logits,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": traffic, "kernel": "mqa_logits_paged_kernel<64, false> (mask tails zeroed in-kernel)",
                     "alg_bytes_per_launch": alg, "peak_source": src},
        "e2e": {"value": total_pairs / (ms_e2e * 1e-3) / 1e9, "unit": "G-scores/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e, "steps": e2e_steps,
                "result_matches_graph": bool(ok)},
        "gpu_launches": args.steps * 2,
        "clocks": clk.summary(),
        "device_status": st,
    }
    if world == 1 and not args.no_cpu_baseline:
        rec["cpu_baseline"] = cpu_decode_sample(w)
    return rec


def cpu_decode_sample(w, n_req=8):
    """Oracle (CPU restatement) on the first n_req requests of the same workload."""
    import numpy as np
    import torch

    from oracle import indexer as O

    G = w["group_size"]
    rows = n_req * G
    q = w["q"][:rows].cpu().view(torch.uint8).numpy().reshape(rows, w["heads"], 128)
    kv = w["kv_cache"].cpu().numpy().reshape(w["kv_cache"].shape[0], -1)
    wt = w["weights"][:rows].cpu().numpy()
    lens = w["context_lens"][:rows].cpu().numpy()
    bt = w["block_table"][:rows].cpu().numpy()
    pt = w["page_table_size_1"][:rows].cpu().numpy()
    t0 = time.perf_counter()
    lg, m, _ = O.mqa_logits_paged(q, kv, wt, lens, bt, w["max_context_len"], G)
    O.topk_transform(lg, m, lens, pt)
    dt = time.perf_counter() - t0
    pairs = float(np.asarray(lens, np.int64).sum())
    return {"value": pairs / dt / 1e9, "unit": "G-scores/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"first {n_req} requests ({rows} rows, {int(pairs)} scores) of the same workload, "
                      f"oracle logits + top-k, {dt:.2f} s"}


def run_reference(args):
    """CPU restatement of the reference pipeline on the same config, all host threads."""
    import numpy as np
    import torch

    from hcu_ops.workloads import config1
    from oracle import indexer as O

    torch.set_num_threads(os.cpu_count() or 1)
    w = config1(device="cpu", seed=0)
    G = w["group_size"]
    q = w["q"].view(torch.uint8).numpy().reshape(w["q"].shape[0], w["heads"], 128)
    kv = w["kv_cache"].numpy().reshape(w["kv_cache"].shape[0], -1)
    lens = w["context_lens"].numpy()
    pairs = float(lens.astype(np.int64).sum())

    def step():
        lg, m, _ = O.mqa_logits_paged(q, kv, w["weights"].numpy(), lens, w["block_table"].numpy(),
                                      w["max_context_len"], G)
        O.topk_transform(lg, m, lens, w["page_table_size_1"].numpy())

    steps = min(args.steps, 20)  # each step is the whole config on the CPU (~1-2 s)
    for _ in range(min(args.warmup, 1)):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    v = pairs / dt / 1e9
    return {
        "impl": "reference",
        "metric": "indexer G-scores/s (rows x visible KV tokens / s), decode logits + top-2048",
        "value": v, "unit": "G-scores/s", "n_gpus": 0, "steps": steps, "warmup": min(args.warmup, 1),
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8e4m3 x fp8e4m3 -> fp32", "data": "synthetic (seeded, same generator as the GPU arm)",
        "config": {"workload": "config1: decode 64 req x next_n 2 (128 rows), ctx U[4096,65536], 64 heads x 128",
                   "pairs": int(pairs)},
        "cpu_baseline": {"value": v, "unit": "G-scores/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": "whole config 1 per step (oracle restatement: the reference's kernels are "
                                   "HIP for gfx938 and lightop is closed)"},
        "e2e": {"value": v, "unit": "G-scores/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------------------------------------
# secondary workloads: bench.py --workload decode0 | prefill | dequant | mla_dequant | kstore | mla_kv | cp_prefill
# (2, 3, the 656-byte MLA dequant, and 4).  Inputs that fit in L2 are timed one
# launch at a time with a 256 MB L2 flush between launches (events around the launch only).
# ------------------------------------------------------------------------------------------------
def _timed_iters(fn, iters, flush):
    import torch

    evs = []
    for _ in range(iters):
        if flush is not None:
            flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        evs.append((a, b))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / iters  # ms


def _flusher(dev):
    import torch

    buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    return lambda: buf.zero_()


def _base_record(args, world, metric, value, unit, ms, workload, **cfg):
    return {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp8e4m3 x fp8e4m3 -> fp32", "data": "synthetic (seeded)",
            "config": dict(workload=workload, **cfg)}


def run_decode0(args, world, rank, local):
    import torch

    import hcu_ops
    from hcu_ops.workloads import config0

    dev = torch.device("cuda", local)
    w = config0(device=dev, seed=rank)
    lens, pt, cu = w["context_lens"], w["page_table_size_1"], w["cu_seqlens_q"]

    def step():
        lg, mk = hcu_ops.mqa_logits(w["q"], w["kv_cache"], w["weights"], lens, w["block_table"],
                                    w["max_context_len"], 1, hist_lens=lens)
        return hcu_ops.sparse_mask_topk_transform(lg, mk, lens, pt, cu, 2048)

    for _ in range(max(args.warmup, 3)):
        step()
    flush = _flusher(dev)
    iters = min(args.steps, 500)
    ms = _timed_iters(step, iters, flush)
    pairs = int(lens.long().sum())
    hbm, _, src = _peaks()
    alg = decode_alg_bytes(w)
    rec = _base_record(args, world, "decode indexer latency, config 0 (1 row x 8192 tokens, 64 heads)",
                       ms * 1e3, "us", ms, "config0: decode 1 x 8192, 64 heads, permuted pages; L2 flushed",
                       pairs=pairs)
    rec["higher_is_better"] = False
    rec["g_scores_per_s"] = pairs / (ms * 1e-3) / 1e9
    rec["roofline"] = {"bound": "latency", "achieved": alg / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                       "frac": alg / (ms * 1e-3) / 1e9 / hbm, "traffic": None, "peak_source": src,
                       "note": "1.1 MB of work: latency-bound, roofline not claimed"}
    rec["gpu_launches"] = iters * 2
    return rec


def run_dequant(args, world, rank, local, mla=False):
    import torch

    import hcu_ops
    from hcu_ops.workloads import make_index_k_dequant, make_mla_dequant

    dev = torch.device("cuda", local)
    if mla:
        n = int(os.environ.get("HCU_BENCH_MLA_TOKENS", "392832"))
        w = make_mla_dequant(n, 1 << 19, seed=rank, device=dev)
        fn = lambda: hcu_ops.dequantize_k_cache_paged(w["quant_k_cache"], w["page_table_1_flattened"])  # noqa: E731
        per_tok = 656 + 1152 + 4
        name = f"MLA 656-byte paged dequant, {n} tokens (pool 2^19 slots)"
    else:
        n = 131072
        w = make_index_k_dequant(n, 4096, seed=rank, device=dev)
        fn = lambda: hcu_ops.dequant_index_k_paged(w["kv_cache"], w["token_loc"])  # noqa: E731
        per_tok = 132 + 256 + 4
        name = "config3: indexer-K paged dequant, 131072 tokens over permuted 64-token pages"
    for _ in range(max(args.warmup, 3)):
        fn()
    iters = min(args.steps, 500)
    ms = _timed_iters(fn, iters, _flusher(dev))
    alg = per_tok * n
    gbs = alg / (ms * 1e-3) / 1e9
    hbm, _, src = _peaks()
    rec = _base_record(args, world, "paged K-cache dequant throughput (algorithmic bytes / s)", gbs * world,
                       "GB/s", ms, name + "; L2 flushed between launches", tokens=n, bytes_per_token=per_tok)
    rec["dtype"] = "fp8e4m3 -> fp32 -> bf16"
    rec["roofline"] = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                       "traffic": None, "alg_bytes_per_launch": alg, "peak_source": src}
    rec["gpu_launches"] = iters
    return rec


def run_kstore(args, world, rank, local):
    """Indexer-K cache writer: 131072 bf16 K rows quantised into permuted slots of a 4096-page pool."""
    import torch

    import hcu_ops

    dev = torch.device("cuda", local)
    n, pool_pages = 131072, 4096
    g = torch.Generator(device=dev)
    g.manual_seed(rank)
    k = torch.randn(n, 128, generator=g, device=dev).to(torch.bfloat16)
    loc = torch.randperm(pool_pages * 64, generator=g, device=dev)[:n].to(torch.int32)
    pool = torch.zeros(pool_pages, 64, 1, 132, dtype=torch.uint8, device=dev)
    fn = lambda: hcu_ops.quant_store_index_k(k, loc, pool)  # noqa: E731
    for _ in range(max(args.warmup, 3)):
        fn()
    iters = min(args.steps, 500)
    ms = _timed_iters(fn, iters, _flusher(dev))
    per_tok = 256 + 4 + 132
    alg = per_tok * n
    gbs = alg / (ms * 1e-3) / 1e9
    hbm, _, src = _peaks()
    rec = _base_record(args, world, "indexer-K cache writer throughput (algorithmic bytes / s)", gbs * world, "GB/s",
                       ms, "indexer-K writer: 131072 bf16 rows -> fp8 + scale into permuted slots of 4096 pages; "
                       "L2 flushed between launches", tokens=n, bytes_per_token=per_tok)
    rec["dtype"] = "bf16 -> fp32 -> fp8e4m3"
    rec["roofline"] = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                       "traffic": None, "alg_bytes_per_launch": alg, "peak_source": src}
    rec["gpu_launches"] = iters
    return rec


MLA_T, MLA_H = 128, 64  # decode tokens of one MLA front-end call, q heads
MLA_BYTES_PER_TOKEN = 2 * MLA_H * 64 * 2 + 2 * 512 * 2 + 2 * 64 * 2 + 128 + 656 + 16  # q, latent, k_pe rw; cos/sin; slot


def _mla_inputs(dev, T, seed):
    """The reference test's layout (hcu_ops/tests/test_kv_fused.py:18-46): a packed [T, 2048 + 576]
    latent, q [T, 64, 256] with the rope tail at 192, a 70000-position cos/sin cache, 4096 slots."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    packed = torch.randn(T, 2048 + 576, generator=g, device=dev).bfloat16()
    q = torch.randn(T, MLA_H, 256, generator=g, device=dev).bfloat16()
    pos = torch.randint(0, 70000, (T,), generator=g, device=dev)
    ang = torch.arange(70000, device=dev)[:, None] * (10000.0 ** (-torch.arange(32, device=dev) / 32))
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).bfloat16().contiguous()
    w = (torch.rand(512, generator=g, device=dev) * 2).bfloat16()
    loc = torch.randperm(4096, generator=g, device=dev)[:T].contiguous()
    buf = torch.zeros(4096, 1, 656, dtype=torch.uint8, device=dev)
    return packed, q, pos, cache, w, loc, buf


def run_mla_kv(args, world, rank, local):
    """MLA decode front end (rope_qout_kv_store): 128 tokens x 64 q heads per call, q rotated in place."""
    import torch

    import hcu_ops

    dev = torch.device("cuda", local)
    packed, q, pos, cache, w, loc, buf = _mla_inputs(dev, MLA_T, rank)
    kv_c, k_pe, q_pe = packed[:, 2048:2560], packed[:, 2560:].unsqueeze(1), q[..., 192:]
    fn = lambda: hcu_ops.rope_qout_kv_store(pos, q_pe, q_pe, kv_c, w, 1e-6, k_pe, cache, False, buf, loc)  # noqa
    for _ in range(max(args.warmup, 3)):
        fn()
    iters = min(args.steps, 500)
    ms = _timed_iters(fn, iters, _flusher(dev))
    alg = MLA_BYTES_PER_TOKEN * MLA_T + 1024
    gbs = alg / (ms * 1e-3) / 1e9
    hbm, _, src = _peaks()
    rec = _base_record(args, world, "MLA decode front end latency (us per call, 128 tokens x 64 q heads)",
                       ms * 1e3, "us", ms, "MLA front end: q rope (64 heads), latent RMS norm in place, k rope, fp8 "
                       "656-byte slot store, 128 decode tokens; L2 flushed between launches", tokens=MLA_T,
                       bytes_per_token=MLA_BYTES_PER_TOKEN)
    rec["higher_is_better"] = False
    rec["dtype"] = "bf16 -> fp32 -> bf16 / fp8e4m3"
    rec["roofline"] = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                       "traffic": None, "alg_bytes_per_launch": alg, "peak_source": src}
    rec["gpu_launches"] = iters
    return rec


def _prefill_inputs(dev, rows, prefix, seed):
    from hcu_ops.workloads import make_ragged

    return make_ragged(rows, prefix, heads=64, seed=seed, device=dev)


def run_prefill(args, world, rank, local):
    import torch

    import hcu_ops

    dev = torch.device("cuda", local)
    p_rows, p_prefix = (8192, 65536) if not args.prefill_shape else args.prefill_shape
    w = _prefill_inputs(dev, p_rows, p_prefix, seed=rank)
    N = w["k_fp8"].shape[0]
    rows = w["q"].shape[0]
    lens = w["row_end"]
    ident = torch.arange(N, dtype=torch.int32, device=dev).expand(rows, N)
    cu = torch.arange(rows + 1, dtype=torch.int32, device=dev)

    def logits():
        return hcu_ops.mqa_logits_ragged(w["q"], w["k_fp8"], w["k_scale"], w["weights"], w["row_start"], lens)

    def step():
        lg, mk = logits()
        return hcu_ops._C.sparse_mask_topk_transform(lg, mk, lens, ident, cu, 2048)

    for _ in range(max(min(args.warmup, 3), 1)):
        step()
    iters = min(args.steps, 10)
    ms = _timed_iters(step, iters, None)
    ms_lg = _timed_iters(logits, iters, None)
    pairs = int((lens.long() - w["row_start"].long()).sum())
    flops = 2.0 * 64 * 128 * pairs
    _, bf16, src = _peaks()
    fp8_peak = 2.0 * bf16
    tflops = flops / (ms_lg * 1e-3) / 1e12
    rec = _base_record(args, world, "prefill indexer G-scores/s (rows x visible KV tokens / s), logits + top-2048",
                       pairs / (ms * 1e-3) / 1e9 * world, "G-scores/s", ms,
                       (f"config2: prefill chunk {rows} rows x ({p_prefix} + i + 1) tokens, 64 heads; "
                        + ("inputs 77 MB, logits 2.4 GB > L2" if not args.prefill_shape else "reduced shape (profiling)")),
                       pairs=pairs)
    rec["logits_op_ms"] = ms_lg
    rec["top_k_rows_per_s"] = rows / ((ms - ms_lg) * 1e-3)
    rec["roofline"] = {"bound": "tensor", "achieved": tflops, "peak": fp8_peak, "unit": "TFLOP/s",
                       "frac": tflops / fp8_peak, "traffic": None, "kernel": "mqa_logits_ragged_kernel<64>",
                       "flops_per_launch": flops, "peak_source": src + " (fp8 dense = 2 x measured bf16 burst)"}
    rec["gpu_launches"] = iters * 2
    return rec


def run_cp_prefill(args, world, rank, local):
    import torch

    from hcu_ops.cp import cp_prefill_topk, kv_range

    dev = torch.device("cuda", local)
    rows, prefix = 16384, 131072 - 16384
    w = _prefill_inputs(dev, rows, prefix, seed=0)  # identical on every rank (replicated q, full K generated)
    N = w["k_fp8"].shape[0]
    lo, hi = kv_range(rank, world, N, causal_rows=rows)  # ranges balanced by visible pairs
    kf = w["k_fp8"][lo:hi].contiguous()
    ks = w["k_scale"][lo:hi].contiguous()
    del w["k_fp8"], w["k_scale"]
    torch.cuda.empty_cache()

    def step():
        return cp_prefill_topk(w["q"], kf, ks, w["weights"], w["row_end"], N, causal_rows=rows)

    for _ in range(max(min(args.warmup, 2), 1)):
        out = step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    iters = min(args.steps, 5)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        out = step()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = t.item()
    pairs = int(w["row_end"].long().sum())
    del out
    if rank != 0:
        return None
    flops = 2.0 * 64 * 128 * pairs
    _, bf16, src = _peaks()
    rec = _base_record(args, world, "CP prefill indexer G-scores/s (rows x visible KV tokens / s), logits + local "
                       "top-2048 + exchange + merge", pairs / (ms * 1e-3) / 1e9, "G-scores/s", ms,
                       "config4: 16384 rows x (114688 + i + 1) tokens over a 131072-token context split into "
                       f"{world} contiguous KV ranges, 64 heads; row-sharded NCCL exchange", pairs=pairs,
                       parallelism=f"cp{world}")
    rec["scaling"] = "strong"
    achieved = flops / (ms * 1e-3) / 1e12
    rec["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": 2.0 * bf16 * world, "unit": "TFLOP/s",
                       "frac": achieved / (2.0 * bf16 * world), "traffic": None,
                       "peak_source": src + " (fp8 dense = 2 x measured bf16 burst, x n_gpus)"}
    rec["gpu_launches"] = iters * 3
    return rec


WORKLOADS = {"decode0": run_decode0, "dequant": run_dequant, "kstore": run_kstore, "mla_kv": run_mla_kv,
             "mla_dequant": lambda a, w, r, l: run_dequant(a, w, r, l, mla=True),
             "prefill": run_prefill, "cp_prefill": run_cp_prefill}


def run_reference_sample(args):
    """CPU oracle on a bounded sample of a secondary workload (--impl reference)."""
    import numpy as np
    import torch

    from oracle import indexer as O

    torch.set_num_threads(os.cpu_count() or 1)
    wl = args.workload
    t0 = time.perf_counter()
    if wl == "decode0":
        from hcu_ops.workloads import config0

        w = config0()
        lg, m, _ = O.mqa_logits_paged(w["q"].view(torch.uint8).numpy().reshape(1, 64, 128),
                                      w["kv_cache"].numpy().reshape(w["kv_cache"].shape[0], -1),
                                      w["weights"].numpy(), w["context_lens"].numpy(), w["block_table"].numpy(),
                                      w["max_context_len"], 1)
        O.topk_transform(lg, m, w["context_lens"].numpy(), w["page_table_size_1"].numpy())
        dt = time.perf_counter() - t0
        value, unit, sample = dt * 1e6, "us", "whole config 0"
    elif wl == "kstore":
        n, pool_pages = 131072, 4096
        g = torch.Generator().manual_seed(0)
        k = torch.randn(n, 128, generator=g).to(torch.bfloat16).float().numpy()
        loc = torch.randperm(pool_pages * 64, generator=g)[:n].to(torch.int32).numpy()
        pool = np.zeros((pool_pages, 64 * 132), np.uint8)
        t0 = time.perf_counter()
        O.quant_store_index_k(k, loc, pool)
        dt = time.perf_counter() - t0
        value, unit, sample = n * (256 + 4 + 132) / dt / 1e9, "GB/s", f"{n} tokens (whole workload)"
    elif wl == "mla_kv":
        from oracle import mla as M

        packed, q, pos, cache, w, loc, buf = _mla_inputs(torch.device("cpu"), MLA_T, 0)
        u = lambda x: x.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        t0 = time.perf_counter()
        M.rope_qout_kv_store(pos.numpy(), u(q[..., 192:]), u(packed[:, 2048:2560]), u(w), 1e-6, u(packed[:, 2560:]),
                             u(cache), False, buf.numpy(), loc.numpy())
        dt = time.perf_counter() - t0
        value, unit, sample = dt * 1e6, "us", f"one call, {MLA_T} tokens x {MLA_H} q heads (whole workload)"
    elif wl in ("dequant", "mla_dequant"):
        from hcu_ops.workloads import make_index_k_dequant, make_mla_dequant

        if wl == "dequant":
            w = make_index_k_dequant(131072, 4096)
            t0 = time.perf_counter()
            O.dequant_index_k(w["kv_cache"].numpy().reshape(4096, -1), w["token_loc"].numpy())
            n, per = 131072, 392
        else:
            w = make_mla_dequant(32768, 1 << 19)
            t0 = time.perf_counter()
            O.dequant_mla_656(w["quant_k_cache"].view(torch.uint8).numpy().reshape(-1, 656),
                              w["page_table_1_flattened"].numpy())
            n, per = 32768, 1812
        dt = time.perf_counter() - t0
        value, unit, sample = n * per / dt / 1e9, "GB/s", f"{n} tokens"
    else:
        rows, prefix = (8192, 65536) if wl == "prefill" else (16384, 131072 - 16384)
        from hcu_ops.workloads import make_ragged

        w = make_ragged(rows, prefix, heads=64)
        sel = np.linspace(0, rows - 1, 64).astype(int)  # stratified subset of rows
        t0 = time.perf_counter()
        lg, m, _ = O.mqa_logits_ragged(w["q"].view(torch.uint8).numpy(), w["k_fp8"].view(torch.uint8).numpy(),
                                       w["k_scale"].numpy(), w["weights"].numpy(), w["row_start"].numpy(),
                                       w["row_end"].numpy(), rows=list(sel))
        N = lg.shape[1]
        O.topk_transform(lg, m, w["row_end"].numpy()[sel], np.tile(np.arange(N, dtype=np.int32), (64, 1)))
        dt = time.perf_counter() - t0
        pairs_s = float(w["row_end"].numpy()[sel].astype(np.int64).sum())
        value, unit = pairs_s / dt / 1e9, "G-scores/s"
        sample = f"64 stratified rows of {rows} ({int(pairs_s)} scores), rate extrapolated by pair count"
    return {"impl": "reference", "metric": f"{wl} (CPU oracle)", "value": value, "unit": unit, "n_gpus": 0,
            "steps": 1, "warmup": 0, "ms_per_step": dt * 1e3, "higher_is_better": unit != "us",
            "config": {"workload": wl},
            "cpu_baseline": {"value": value, "unit": unit, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill-shape", type=int, nargs=2, metavar=("ROWS", "PREFIX"), default=None,
                    help="prefill workload at a reduced shape (for profiler captures); default config 2")
    args = ap.parse_args()
    world, rank, local = _dist()
    if args.impl == "reference":
        if rank == 0:
            rec = run_reference(args) if args.workload == "decode" else run_reference_sample(args)
            print(json.dumps(rec), flush=True)
        return
    import torch

    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    try:
        if args.workload == "decode":
            rec = run_decode(args, world, rank, local)
        elif args.workload in WORKLOADS:
            rec = WORKLOADS[args.workload](args, world, rank, local)
            if rec is not None and world > 1 and args.workload != "cp_prefill":
                rec = rec if rank == 0 else None
        else:
            raise SystemExit(f"unknown workload {args.workload}")
        if rec is not None:
            print(json.dumps(rec), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
