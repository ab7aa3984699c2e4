#!/usr/bin/env python
"""Benchmark of the DSA lightning-indexer path on B200.

Headline (the decode indexer the metric is quoted on): 64 requests x next_n=2
rows, contexts U[4096, 65536], 64 index heads x 128 dim fp8, shared shuffled pool of 64-token pages.
One step = one CUDA-graph replay of the sglang decode call pair: hcu_ops.mqa_logits (tcgen05 fp8
paged logits + mask) -> hcu_ops.sparse_mask_topk_transform (exact top-2048 + page-table transform).
metric: G-scores/s = (sum over rows of visible KV tokens) / step time.  The decode indexer does not
shard: under torchrun every rank runs its own replica ("scaling": "weak"); value = all ranks' scores /
the slowest rank's time.  A stratified row sample of the headline step is checked against the CPU
oracle in the same run ("oracle_check").

Sub-records of the same JSON line:
  cp_prefill  config 4 of BASELINE.json at this N (every N, 1 included): 16384 rows over a 131072-token
              context split into N KV ranges (hcu_ops.cp); per-rank time spread, clocks, list length,
              reruns, and equality with the one-range result computed on rank 0.
  secondary   (N = 1) configs 0, 2, 3, the 656-byte MLA dequant, the indexer-K writer and the MLA
              front end, each with its roofline, clocks and CPU baseline.

--impl reference: the CPU restatement of the reference's algorithm (the reference's kernels are HIP
for gfx938 and its oracle library is closed) on the host cores, rank 0 only, same metric, config,
steps and warm-up; it loads none of this repository's compiled libraries.
--workload NAME runs one secondary workload alone (decode0, prefill, dequant, mla_dequant, kstore,
mla_kv, cp_filter, cp_prefill).
"""
from __future__ import annotations

import argparse
import importlib.util
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
METRIC = "indexer G-scores/s (rows x visible KV tokens / s), decode logits + top-2048"
DTYPE = "fp8e4m3 x fp8e4m3 -> fp32"


def _workloads():
    """The seeded input generators, loaded by path so that no compiled library is imported."""
    spec = importlib.util.spec_from_file_location("hcu_workloads",
                                                  os.path.join(PKG_ROOT, "hcu_ops", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


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
        self.out = ""

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def __exit__(self, *a):
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


def _events():
    import torch

    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _timed(fn, steps, local):
    """steps calls of fn on the current stream between CUDA events (synchronised on both sides),
    clocks sampled meanwhile; returns (ms per call, clocks)."""
    import torch

    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        a, b = _events()
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
    return a.elapsed_time(b) / steps, clk.summary()


def _read_flush(dev):
    """An L2 flush that leaves no dirty lines behind: a reduction reading 256 MB."""
    import torch

    buf = torch.ones(256 << 20, dtype=torch.uint8, device=dev)
    return lambda: buf.sum(dtype=torch.int32)


def _per_launch(fn, iters, flush, local):
    """Mean time of single launches, each after an L2 flush (events around the launch only)."""
    import torch

    evs = []
    with ClockSampler(local) as clk:
        for _ in range(iters):
            flush()
            a, b = _events()
            a.record()
            fn()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / iters, clk.summary()


# ------------------------------------------------------------------------------------------------
# headline: decode (config 1)
# ------------------------------------------------------------------------------------------------
def decode_alg_bytes(w):
    """Algorithmic HBM bytes of one logits launch: each group's K pages read once (128 fp8 + 4 B
    scale per token), q + weights, block-table entries, logits written at every visible token,
    and the mask words of the full width (each processed tile's words, the rest zeroed by the kernel)."""
    lens = w["context_lens"].long().cpu()
    G, H = w["group_size"], w["heads"]
    B = lens.numel()
    glen = lens.view(-1, G).max(1).values
    k_bytes = int((glen * 132).sum())
    bt_bytes = int(((glen + 63) // 64).sum() * 4)
    q_bytes = B * H * 128 + B * H * 4
    logits_bytes = int(lens.sum() * 4)
    mask_bytes = B * (w["max_context_len"] // 16) * 2 + int(((glen + 127) // 128).sum() * G * 16)
    return k_bytes + bt_bytes + q_bytes + logits_bytes + mask_bytes


def decode_config(world, seed=0):
    """The headline's `config` (identical in both arms); computed from the generator's lengths."""
    wl = _workloads()
    lens = wl.config1_lens(seed)
    pages = sum((L + 63) // 64 for L in lens)
    return {"workload": "config1: decode 64 req x next_n 2 (128 rows), ctx U[4096,65536], 64 heads x 128, "
                        "64-token pages, shuffled pool; CUDA-graph replay",
            "rows": 2 * len(lens), "heads": 64, "width": 65536, "pairs_per_gpu": sum(2 * L - 1 for L in lens),
            "kv_pool_bytes": pages * 64 * 132, "l2": "no flush: K pool > 126 MB L2",
            "parallelism": f"replicas x{world}"}


def decode_oracle_check(w, lg, mk, out, n_req=8):
    """The oracle on the first n_req requests of the step's inputs, against the device's logits, mask
    and selection: (check dict, CPU seconds of the oracle's logits + top-k)."""
    import numpy as np
    import torch

    from oracle import indexer as O

    G = w["group_size"]
    rows = n_req * G
    W = w["max_context_len"]
    q = w["q"][:rows].cpu().view(torch.uint8).numpy().reshape(rows, w["heads"], 128)
    kv = w["kv_cache"].cpu().numpy().reshape(w["kv_cache"].shape[0], -1)
    lens = w["context_lens"][:rows].cpu().numpy()
    pt = w["page_table_size_1"][:rows].cpu().numpy()
    t0 = time.perf_counter()
    rl, rm, fl = O.mqa_logits_paged(q, kv, w["weights"][:rows].cpu().numpy(), lens, w["block_table"][:rows].cpu().numpy(),
                                    W, G, want_floor=True)
    ref = O.topk_transform(rl, rm, lens, pt)
    dt = time.perf_counter() - t0
    dl, dm, do = lg[:rows].cpu().numpy(), mk[:rows].cpu().numpy(), out[:rows].cpu().numpy()
    md, mr = O.mask_bits(dm, W), O.mask_bits(rm, W)
    both = md & mr
    rel = np.abs(dl[both] - rl[both]) / np.maximum(np.abs(rl[both]), fl[both])
    same = O.topk_transform(dl, dm, lens, pt)
    ov = np.mean([len(set(a[a >= 0].tolist()) & set(b[b >= 0].tolist())) / max(int((b >= 0).sum()), 1)
                  for a, b in zip(do, ref)])
    chk = {"rows": rows, "logits_max_rel_err": float(rel.max(initial=0.0)), "logits_tol": 1e-2,
           "mask_bits_differing": int((md ^ mr).sum()), "topk_exact_on_device_logits": bool(np.array_equal(do, same)),
           "e2e_overlap": float(ov)}
    chk["ok"] = bool(chk["logits_max_rel_err"] <= 1e-2 and chk["topk_exact_on_device_logits"] and ov >= 0.999)
    return chk, dt, float(np.asarray(lens, np.int64).sum())


def run_decode(args, world, rank, local):
    import torch

    import hcu_ops
    from hcu_ops.workloads import config1

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = config1(device=dev, seed=rank)
    pairs = int(w["context_lens"].long().sum())
    lens, pt, cu = w["context_lens"], w["page_table_size_1"], w["cu_seqlens_q"]

    def step():
        lg, mk = hcu_ops.mqa_logits(w["q"], w["kv_cache"], w["weights"], lens, w["block_table"],
                                    w["max_context_len"], w["group_size"], hist_lens=lens)
        return lg, mk, hcu_ops.sparse_mask_topk_transform(lg, mk, lens, pt, cu, 2048)

    def logits_only():
        return hcu_ops._C.mqa_logits_hist(w["q"], w["kv_cache"], w["weights"], lens, w["block_table"],
                                          w["max_context_len"], w["group_size"], 0, 0, None)

    warm = max(args.warmup, 3)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warm):
            step()
            logits_only()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        lg_g, mk_g, out = step()
    g_lg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_lg):
        logits_only()
    for _ in range(warm):
        g.replay()
        g_lg.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # ---- headline: K graph replays of the pipeline (inputs resident in HBM; the K pool exceeds L2)
    barrier()
    ms, clocks = _timed(g.replay, args.steps, local)
    barrier()
    # ---- the dominant kernel alone (the logits op) for the roofline
    ms_logits, _ = _timed(g_lg.replay, args.steps, local)
    barrier()
    ms_e2e, e2e_steps, h2d, d2h, e2e_ok = _decode_e2e(w, out, args.steps)
    st = hcu_ops.read_device_status(clear=True)

    t = torch.tensor([ms, ms_logits, ms_e2e, float(pairs)], dtype=torch.float64, device=dev)
    per_rank_ms = [ms]
    per_rank_logits = [ms_logits]
    if world > 1:
        allt = [torch.zeros_like(t) for _ in range(world)]
        torch.distributed.all_gather(allt, t)
        per_rank_ms = [float(x[0]) for x in allt]
        per_rank_logits = [float(x[1]) for x in allt]
        ms = max(float(x[0]) for x in allt)
        ms_logits = max(float(x[1]) for x in allt)
        ms_e2e = max(float(x[2]) for x in allt)
        total_pairs = sum(float(x[3]) for x in allt)
    else:
        total_pairs = float(pairs)
    if rank != 0:
        return None
    check, cpu_s, cpu_pairs = decode_oracle_check(w, lg_g, mk_g, out)
    hbm, _, src = _peaks()
    alg = decode_alg_bytes(w)
    achieved = alg / (ms_logits * 1e-3) / 1e9
    rec = {
        "metric": METRIC,
        "value": total_pairs / (ms * 1e-3) / 1e9,
        "unit": "G-scores/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": DTYPE,
        "data": "synthetic (seeded; q,K ~ N(0,1) per-row/per-token amax/448 fp8; w ~ N(0,1)/8)",
        "config": decode_config(world),
        "per_rank_ms": {"min": min(per_rank_ms), "median": statistics.median(per_rank_ms), "max": max(per_rank_ms),
                        "all": per_rank_ms},
        "per_rank_logits_op_ms": {"min": min(per_rank_logits), "median": statistics.median(per_rank_logits),
                                  "max": max(per_rank_logits), "all": per_rank_logits},
        "top_k_rows_per_s": lens.numel() * world / (ms * 1e-3),
        "logits_op_ms": ms_logits,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": _profile_traffic("mqa_logits_paged_config1"),
                     "kernel": "mqa_logits_paged_kernel<64, false> (mask tails zeroed in-kernel)",
                     "alg_bytes_per_launch": alg, "peak_source": src},
        "step_roofline": {"alg_bytes": alg + lens.numel() * 2048 * 8, "frac_of_hbm": (alg + lens.numel() * 2048 * 8)
                          / (ms * 1e-3) / 1e9 / hbm, "note": "logits launch bytes + the top-k's page-table gather "
                                                             "and output"},
        "e2e": {"value": total_pairs / (ms_e2e * 1e-3) / 1e9, "unit": "G-scores/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e, "steps": e2e_steps,
                "result_matches_graph": bool(e2e_ok),
                "how": "public API under CUDA-graph capture (as serving runs it); every step copies its inputs "
                       "(one pinned staging buffer) in and its [128, 2048] result out, on two copy streams, "
                       "double-buffered against the compute"},
        "gpu_launches": args.steps * 2,
        "clocks": clocks,
        "device_status": st,
        "oracle_check": check,
    }
    if world == 1 and not args.no_cpu_baseline:
        rec["cpu_baseline"] = {"value": cpu_pairs / cpu_s / 1e9, "unit": "G-scores/s", "cores": _threads(),
                               "kind": "port",
                               "sample": f"first 8 requests ({check['rows']} rows, {int(cpu_pairs)} scores) of the "
                                         f"same workload, oracle logits + top-k, {cpu_s:.2f} s"}
    return rec


def _threads():
    import torch

    return torch.get_num_threads()


def _decode_e2e(w, out_graph, steps):
    """The headline metric through the public API with host buffers, as a serving engine runs it:
    every step copies its inputs (query rows, head weights, context lengths, block table) from one
    pinned host staging buffer into the device (one copy), replays the CUDA graph of
    hcu_ops.mqa_logits -> hcu_ops.sparse_mask_topk_transform captured over those device inputs, and
    copies the [rows, 2048] result back into pinned host memory.  The KV cache and the per-token page
    table (built on the device by the serving engine's metadata step) are device state.  Two input
    buffers and two captured graphs alternate, so step i + 1's inputs and step i - 1's result cross
    PCIe while step i computes (host->device and device->host on separate copy streams)."""
    import torch

    import hcu_ops

    keys = ("q", "weights", "context_lens", "block_table")
    offs, n = {}, 0
    for k in keys:  # each input at a 256-byte aligned offset of one staging buffer
        offs[k] = n
        n += (w[k].numel() * w[k].element_size() + 255) // 256 * 256
    host = torch.empty(n, dtype=torch.uint8).pin_memory()
    for k in keys:
        nb = w[k].numel() * w[k].element_size()
        host[offs[k]:offs[k] + nb].copy_(w[k].reshape(-1).view(torch.uint8).cpu())
    dev = w["q"].device
    dbuf = [torch.empty(n, dtype=torch.uint8, device=dev) for _ in range(2)]

    def views(buf):
        return {k: buf[offs[k]:offs[k] + w[k].numel() * w[k].element_size()].view(w[k].dtype).view(w[k].shape)
                for k in keys}

    pt, cu, kv, width, G = (w["page_table_size_1"], w["cu_seqlens_q"], w["kv_cache"], w["max_context_len"],
                            w["group_size"])

    def step(d):
        lg, mk = hcu_ops.mqa_logits(d["q"], kv, d["weights"], d["context_lens"], d["block_table"], width, G,
                                    hist_lens=d["context_lens"])
        return hcu_ops.sparse_mask_topk_transform(lg, mk, d["context_lens"], pt, cu, 2048)

    for d in dbuf:
        d.copy_(host)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for d in dbuf:
            for _ in range(2):
                step(views(d))
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graphs, outs, pool = [], [], None
    for d in dbuf:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=pool):
            outs.append(step(views(d)))
        pool = g.pool()
        graphs.append(g)
    rows = w["context_lens"].numel()
    res_host = [torch.empty((rows, 2048), dtype=torch.int32).pin_memory() for _ in range(2)]
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def load(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_done[b])  # step i - 2 no longer reads this input buffer
            dbuf[b].copy_(host, non_blocking=True)
            ev_in[b].record(s_in)

    def run(nsteps):
        load(0)
        for i in range(nsteps):
            b = i % 2
            if i + 1 < nsteps:
                load(i + 1)
            comp.wait_event(ev_in[b])
            if i >= 2:
                comp.wait_event(ev_out[b])  # step i - 2's result has left this output buffer
            graphs[b].replay()
            ev_done[b].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[b])
                res_host[b].copy_(outs[b], non_blocking=True)
                ev_out[b].record(s_out)
        comp.wait_stream(s_out)
        comp.wait_stream(s_in)

    run(4)
    torch.cuda.synchronize()
    nsteps = max(2, min(steps, 200))
    a, b = _events()
    a.record()
    run(nsteps)
    b.record()
    torch.cuda.synchronize()
    ok = torch.equal(res_host[(nsteps - 1) % 2], out_graph.cpu())
    del graphs
    return a.elapsed_time(b) / nsteps, nsteps, n, rows * 2048 * 4, ok


def _decode_ref_sample_reqs(steps, warmup, budget_s=120.0, per_step_s=1.3):
    """Requests per reference step: the whole config when (steps + warm-up) fit the CPU budget,
    else a proportional subset (each step is then a bounded sample of the workload)."""
    n = int(64 * budget_s / max((steps + warmup) * per_step_s, 1e-9))
    return max(1, min(64, n))


def run_reference(args):
    """CPU restatement of the reference pipeline on the headline config, all host threads: logits of
    every visible (row, token) pair and the exact top-2048 of every row, per step."""
    import numpy as np
    import torch

    from oracle import indexer as O

    wl = _workloads()
    world, _, _ = _dist()
    torch.set_num_threads(os.cpu_count() or 1)
    w = wl.config1(device="cpu", seed=0)
    G = w["group_size"]
    n_req = _decode_ref_sample_reqs(args.steps, args.warmup)
    rows = n_req * G
    q = w["q"][:rows].view(torch.uint8).numpy().reshape(rows, w["heads"], 128)
    kv = w["kv_cache"].numpy().reshape(w["kv_cache"].shape[0], -1)
    lens = w["context_lens"][:rows].numpy()
    bt = w["block_table"][:rows].numpy()
    pt = w["page_table_size_1"][:rows].numpy()
    wt = w["weights"][:rows].numpy()
    pairs = float(lens.astype(np.int64).sum())

    def step():
        lg, m, _ = O.mqa_logits_paged(q, kv, wt, lens, bt, w["max_context_len"], G)
        O.topk_transform(lg, m, lens, pt)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    v = pairs / dt / 1e9
    sample = ("whole config 1 per step" if n_req == 64 else
              f"first {n_req} of 64 requests ({rows} rows, {int(pairs)} scores) per step")
    return {
        "impl": "reference",
        "metric": METRIC, "value": v, "unit": "G-scores/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic (seeded, same generator as the GPU arm)",
        "config": decode_config(world),
        "cpu_baseline": {"value": v, "unit": "G-scores/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample + " (CPU restatement of the reference's algorithm: its kernels are HIP "
                                            "for gfx938 and its bit-exact oracle library is closed)"},
        "e2e": {"value": v, "unit": "G-scores/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------------------------------------
# config 4: context-parallel prefill (every N)
# ------------------------------------------------------------------------------------------------
CP_ROWS, CP_N = 16384, 131072


def _stratified(rows, n=64):
    import numpy as np

    return np.unique(np.linspace(0, rows - 1, n).astype(np.int64))


def _ragged_cpu_sample(rows, prefix, topk_too=True):
    """CPU oracle (logits + top-k) on 64 stratified rows of a ragged workload: (G-scores/s, sample text)."""
    import numpy as np
    import torch

    from oracle import indexer as O

    w = _workloads().make_ragged(rows, prefix, heads=64)
    sel = _stratified(rows)
    t0 = time.perf_counter()
    lg, m, _ = O.mqa_logits_ragged(w["q"].view(torch.uint8).numpy(), w["k_fp8"].view(torch.uint8).numpy(),
                                   w["k_scale"].numpy(), w["weights"].numpy(), w["row_start"].numpy(),
                                   w["row_end"].numpy(), rows=list(sel))
    if topk_too:
        N = lg.shape[1]
        O.topk_transform(lg, m, w["row_end"].numpy()[sel], np.broadcast_to(np.arange(N, dtype=np.int32), (len(sel), N)))
    dt = time.perf_counter() - t0
    pairs = float(w["row_end"].numpy()[sel].astype(np.int64).sum())
    return pairs / dt / 1e9, (f"{len(sel)} stratified rows of {rows} ({int(pairs)} scores, {dt:.2f} s), oracle "
                              f"logits + top-k; rate extrapolated to the whole workload by pair count")


def run_cp_prefill(args, world, rank, local, steps=None, warmup=None):
    import torch

    import hcu_ops
    from hcu_ops.cp import calibrate_shares, cp_prefill_topk, kv_range, list_len

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    rows, N = CP_ROWS, CP_N
    # KV ranges balanced by visible pairs, weighted by each GPU's measured prefill-logits rate (GPUs of
    # one box differ; the step waits for the slowest rank).  HCU_CP_SHARES=equal: unweighted.
    shares = None
    if world > 1 and os.environ.get("HCU_CP_SHARES", "calibrated") != "equal":
        shares = calibrate_shares(device=dev)
    w = _workloads().make_ragged(rows, N - rows, heads=64, seed=0, device=dev)  # identical on every rank
    lo, hi = kv_range(rank, world, N, causal_rows=rows, shares=shares)
    kf, ks = w["k_fp8"][lo:hi].contiguous(), w["k_scale"][lo:hi].contiguous()
    steps = steps or min(args.steps, 20)
    warmup = warmup or max(3, min(args.warmup, 5))
    stats = {}

    def step():
        return cp_prefill_topk(w["q"], kf, ks, w["weights"], w["row_end"], N, causal_rows=rows, stats=stats,
                               shares=shares)

    for _ in range(warmup):
        out = step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    stats.clear()
    with ClockSampler(local) as clk:
        a, b = _events()
        a.record()
        for _ in range(steps):
            out = step()
        b.record()
        torch.cuda.synchronize()
    ms_mine = a.elapsed_time(b) / steps
    t = torch.tensor([ms_mine], dtype=torch.float64, device=dev)
    per_rank = [ms_mine]
    if world > 1:
        allt = [torch.zeros_like(t) for _ in range(world)]
        torch.distributed.all_gather(allt, t)
        per_rank = [float(x.item()) for x in allt]
    ms = max(per_rank)
    reruns = stats.get("reruns", 0)
    if world > 1:
        r = torch.tensor([reruns], dtype=torch.int64, device=dev)
        torch.distributed.all_reduce(r, op=torch.distributed.ReduceOp.MAX)
        reruns = int(r.item())
    if rank != 0:
        return None
    # the one-range result on this GPU (untimed equality check), then its time on the same box
    ident = torch.arange(N, dtype=torch.int32, device=dev).expand(rows, N)
    cu = torch.arange(rows + 1, dtype=torch.int32, device=dev)
    zeros = torch.zeros(rows, dtype=torch.int32, device=dev)

    def one_gpu():
        lg, mk = hcu_ops.mqa_logits_ragged(w["q"], w["k_fp8"], w["k_scale"], w["weights"], zeros, w["row_end"])
        return hcu_ops.sparse_mask_topk_transform(lg, mk, w["row_end"], ident, cu, 2048)

    ref = one_gpu()
    matches = bool(torch.equal(out, ref))
    del ref
    ms_one = None
    if world > 1:
        one_gpu()
        ms_one, _ = _timed(one_gpu, 3, local)
    pairs = int(w["row_end"].long().sum())
    flops = 2.0 * 64 * 128 * pairs
    _, bf16, src = _peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    rec = {"metric": "CP prefill indexer G-scores/s (rows x visible KV tokens / s): logits + bounds + filter + "
                     "exchange + merge", "value": pairs / (ms * 1e-3) / 1e9, "unit": "G-scores/s", "n_gpus": world,
           "steps": steps, "warmup": warmup, "ms_per_step": ms, "scaling": "strong",
           "per_rank_ms": {"min": min(per_rank), "median": statistics.median(per_rank), "max": max(per_rank)},
           "config": {"workload": f"config4: {rows} rows x ({N - rows} + i + 1) tokens over a {N}-token context in "
                                  f"{world} KV ranges balanced by visible pairs" +
                                  (", weighted by each GPU's measured logits rate" if shares else "") + ", 64 heads",
                      "pairs": pairs, "shares": [round(x / max(shares), 4) for x in shares] if shares else None,
                      "parallelism": f"cp{world}", "l2": "no flush: logits and inputs exceed L2"},
           "list_len": list_len(world) if world > 1 else None, "reruns": reruns,
           "exchange": stats.get("exchange", "none (one range)"),
           "matches_1gpu": matches,
           "roofline": {"bound": "tensor", "achieved": achieved, "peak": 2.0 * bf16 * world, "unit": "TFLOP/s",
                        "frac": achieved / (2.0 * bf16 * world), "traffic": None,
                        "peak_source": src + " (fp8 dense = 2 x measured bf16 burst, x n_gpus)"},
           "gpu_launches_per_step": stats.get("launches"),
           "clocks": clk.summary()}
    if ms_one is not None:
        rec["one_gpu_ms_same_box"] = ms_one
        rec["speedup_vs_one_gpu"] = ms_one / ms
    if world == 1 and not args.no_cpu_baseline:
        v, sample = _ragged_cpu_sample(rows, N - rows)
        rec["cpu_baseline"] = {"value": v, "unit": "G-scores/s", "cores": _threads(), "kind": "port",
                               "sample": sample}
    return rec


# ------------------------------------------------------------------------------------------------
# secondary workloads (N = 1): configs 0, 2, 3, the 656-byte MLA dequant, the K writer, the MLA front end
# ------------------------------------------------------------------------------------------------
def _rec(metric, value, unit, ms, steps, workload, higher=True, **cfg):
    return {"metric": metric, "value": value, "unit": unit, "ms_per_step": ms, "steps": steps,
            "higher_is_better": higher, "config": dict(workload=workload, **cfg)}


def _rotating_graph(fns, launches, dev):
    """A CUDA graph of `launches` calls cycling through the instances' callables (their inputs
    together exceed L2); every launch's output stays allocated, so each writes its own buffer and
    every launch streams from and to HBM.  Returns (graph, the outputs it writes)."""
    import torch

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    keep = []
    with torch.cuda.graph(g):
        for i in range(launches):
            keep.append(fns[i % len(fns)]())
    return g, keep


def _hbm_loop(fns, per_launch_bytes, steps, local, dev):
    """Graph-replayed back-to-back launches over rotating instances: (ms per launch, clocks, launches)."""
    per_graph = 4 * len(fns)
    g, keep = _rotating_graph(fns, per_graph, dev)
    for _ in range(3):
        g.replay()
    reps = max(1, min(steps, 50))
    ms, clocks = _timed(g.replay, reps, local)
    del keep
    return ms / per_graph, clocks, reps * per_graph


def _instances(bytes_per_instance):
    return max(2, -(-3 * L2_BYTES // max(bytes_per_instance, 1)))


def sec_decode0(args, local):
    import torch

    import hcu_ops

    dev = torch.device("cuda", local)
    wl = _workloads()
    w = wl.config0(device=dev, seed=0)
    lens, pt, cu = w["context_lens"], w["page_table_size_1"], w["cu_seqlens_q"]

    def step():
        lg, mk = hcu_ops.mqa_logits(w["q"], w["kv_cache"], w["weights"], lens, w["block_table"],
                                    w["max_context_len"], 1, hist_lens=lens)
        return hcu_ops.sparse_mask_topk_transform(lg, mk, lens, pt, cu, 2048)

    for _ in range(5):
        step()
    iters = max(10, min(args.steps, 200))
    ms, clocks = _per_launch(step, iters, _read_flush(dev), local)
    pairs = int(lens.long().sum())
    hbm, _, src = _peaks()
    alg = decode_alg_bytes(w)
    rec = _rec("decode indexer latency, config 0 (1 row x 8192 tokens, 64 heads), logits + top-2048", ms * 1e3,
               "us", ms, iters, "config0: decode 1 x 8192, 64 heads, permuted pages; L2 flushed (read) before "
               "every call", higher=False, pairs=pairs)
    rec["roofline"] = {"bound": "latency", "achieved": alg / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                       "frac": alg / (ms * 1e-3) / 1e9 / hbm, "traffic": None, "peak_source": src,
                       "note": "1.1 MB of work: latency-bound, roofline not claimed"}
    rec["gpu_launches"] = iters * 3
    rec["clocks"] = clocks
    if not args.no_cpu_baseline:
        import numpy as np

        from oracle import indexer as O

        wc = wl.config0()
        t0 = time.perf_counter()
        lg, m, _ = O.mqa_logits_paged(wc["q"].view(torch.uint8).numpy().reshape(1, 64, 128),
                                      wc["kv_cache"].numpy().reshape(wc["kv_cache"].shape[0], -1),
                                      wc["weights"].numpy(), wc["context_lens"].numpy(), wc["block_table"].numpy(),
                                      wc["max_context_len"], 1)
        O.topk_transform(lg, m, wc["context_lens"].numpy(), wc["page_table_size_1"].numpy())
        dt = time.perf_counter() - t0
        rec["cpu_baseline"] = {"value": dt * 1e6, "unit": "us", "cores": _threads(), "kind": "port",
                               "sample": "whole config 0 (oracle logits + top-k)"}
        del np
    return rec


def sec_prefill(args, local):
    """Config 2: logits + top-k of a 8192-row prefill chunk over a 65536-token prefix."""
    import torch

    import hcu_ops

    dev = torch.device("cuda", local)
    p_rows, p_prefix = (8192, 65536) if not args.prefill_shape else args.prefill_shape
    w = _workloads().make_ragged(p_rows, p_prefix, heads=64, seed=0, device=dev)
    N = w["k_fp8"].shape[0]
    rows = w["q"].shape[0]
    lens = w["row_end"]
    ident = torch.arange(N, dtype=torch.int32, device=dev).expand(rows, N)
    cu = torch.arange(rows + 1, dtype=torch.int32, device=dev)
    state = {}

    def logits():
        state["lg"] = hcu_ops.mqa_logits_ragged(w["q"], w["k_fp8"], w["k_scale"], w["weights"], w["row_start"], lens)

    def topk():
        lg, mk = state["lg"]
        return hcu_ops.sparse_mask_topk_transform(lg, mk, lens, ident, cu, 2048)

    def step():
        logits()
        return topk()

    flag = torch.zeros(1, dtype=torch.int32, device=dev)

    def fused():
        return hcu_ops.mqa_topk_ragged(w["q"], w["k_fp8"], w["k_scale"], w["weights"], lens, ident, fallback_flag=flag)

    for _ in range(3):
        ref = step()
        got = fused()
    fused_equal = bool(torch.equal(got, ref))
    del ref, got
    iters = max(3, min(args.steps, 10))
    ms_pair, _ = _timed(step, iters, local)
    ms_lg, _ = _timed(logits, iters, local)
    ms_tk, _ = _timed(topk, iters, local)
    state.clear()
    torch.cuda.empty_cache()
    ms_fused, clocks = _timed(fused, iters, local)
    fell_back = int(flag.item())
    ms = min(ms_pair, ms_fused)  # the record's value: the faster of the two public paths
    pairs = int((lens.long() - w["row_start"].long()).sum())
    flops = 2.0 * 64 * 128 * pairs
    hbm, bf16, src = _peaks()
    fp8_peak = 2.0 * bf16
    tflops = flops / (ms_lg * 1e-3) / 1e12
    shape = "config2" if not args.prefill_shape else "reduced shape (profiling)"
    rec = _rec("prefill indexer G-scores/s (rows x visible KV tokens / s), logits + top-2048",
               pairs / (ms * 1e-3) / 1e9, "G-scores/s", ms, iters,
               f"{shape}: prefill chunk {rows} rows x ({p_prefix} + i + 1) tokens, 64 heads; the faster of "
               f"the materialised pair and the fused hcu_ops.mqa_topk_ragged; inputs > L2, no flush", pairs=pairs)
    rec["path"] = "fused" if ms_fused <= ms_pair else "materialised_pair"
    rec["fused"] = {"ms": ms_fused, "value": pairs / (ms_fused * 1e-3) / 1e9,
                    "equals_materialised_pair": fused_equal, "exact_path_ran": fell_back,
                    "how": "sampled bound (1/64 of K) -> logits appending tokens at or above it to per-row "
                           "lists -> select; exact materialising path predicated on a device flag"}
    rec["materialised_pair"] = {"ms": ms_pair, "value": pairs / (ms_pair * 1e-3) / 1e9,
                                "logits_bytes": rows * N * 4,
                                "how": "mqa_logits_ragged (logits + mask in HBM) -> sparse_mask_topk_transform"}
    rec["logits_op_ms"] = ms_lg
    rec["topk_op_ms"] = ms_tk
    rec["top_k_rows_per_s"] = rows / (ms_tk * 1e-3)
    topk_bytes = rows * N * 4 + rows * (N // 16) * 2 + rows * 2048 * 8
    rec["topk_roofline"] = {"bound": "hbm", "achieved": topk_bytes / (ms_tk * 1e-3) / 1e9, "peak": hbm,
                            "unit": "GB/s", "frac": topk_bytes / (ms_tk * 1e-3) / 1e9 / hbm}
    rec["roofline"] = {"bound": "tensor", "achieved": tflops, "peak": fp8_peak, "unit": "TFLOP/s",
                       "frac": tflops / fp8_peak, "traffic": None, "kernel": "mqa_logits_ragged_kernel<64>",
                       "flops_per_launch": flops, "peak_source": src + " (fp8 dense = 2 x measured bf16 burst)"}
    rec["gpu_launches"] = iters * 7  # fused: prep, sampled logits, bound, logits, select, two predicated
    rec["clocks"] = clocks
    if not args.no_cpu_baseline and not args.prefill_shape:
        v, sample = _ragged_cpu_sample(p_rows, p_prefix)
        rec["cpu_baseline"] = {"value": v, "unit": "G-scores/s", "cores": _threads(), "kind": "port",
                               "sample": sample}
    return rec


def sec_dequant(args, local, mla=False):
    """Config 3 (indexer-K pages -> bf16) or the 656-byte MLA slots -> bf16, HBM-bound: back-to-back
    graph-replayed launches over enough rotating instances that every launch streams from HBM."""
    import numpy as np
    import torch

    import hcu_ops

    dev = torch.device("cuda", local)
    wl = _workloads()
    if mla:
        n = int(os.environ.get("HCU_BENCH_MLA_TOKENS", "392832"))
        per_tok = 656 + 1152 + 4
        inst = [wl.make_mla_dequant(n, 1 << 19, seed=i, device=dev) for i in range(2)]
        fns = [lambda m=m: hcu_ops.dequantize_k_cache_paged(m["quant_k_cache"], m["page_table_1_flattened"])
               for m in inst]
        name = f"MLA 656-byte paged dequant, {n} tokens over a 2^19-slot pool"
        kernel = "dequant_mla_kernel"
    else:
        n = 131072
        per_tok = 132 + 256 + 4
        k = _instances(n * per_tok)
        inst = [wl.make_index_k_dequant(n, 4096, seed=i, device=dev) for i in range(k)]
        fns = [lambda m=m: hcu_ops.dequant_index_k_paged(m["kv_cache"], m["token_loc"]) for m in inst]
        name = f"config3: indexer-K paged dequant, {n} tokens over permuted 64-token pages"
        kernel = "dequant_index_k_kernel"
    alg = per_tok * n
    ms, clocks, launches = _hbm_loop(fns, alg, args.steps, local, dev)
    gbs = alg / (ms * 1e-3) / 1e9
    hbm, _, src = _peaks()
    rec = _rec("paged K-cache dequant throughput (algorithmic bytes / s)", gbs, "GB/s", ms, launches,
               f"{name}; graph-replayed launches cycling {len(fns)} input/output sets "
               f"({len(fns) * alg / 1e6:.0f} MB > L2)", tokens=n, bytes_per_token=per_tok)
    rec["dtype"] = "fp8e4m3 -> fp32 -> bf16"
    rec["roofline"] = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                       "traffic": _profile_traffic(kernel + ("_mla" if mla else "_config3")),
                       "kernel": kernel, "alg_bytes_per_launch": alg, "peak_source": src}
    rec["gpu_launches"] = launches
    rec["clocks"] = clocks
    if not args.no_cpu_baseline:
        from oracle import indexer as O

        if mla:
            m = wl.make_mla_dequant(32768, 1 << 19)
            t0 = time.perf_counter()
            O.dequant_mla_656(m["quant_k_cache"].view(torch.uint8).numpy().reshape(-1, 656),
                              m["page_table_1_flattened"].numpy())
            dt, nn = time.perf_counter() - t0, 32768
        else:
            m = wl.make_index_k_dequant(n, 4096)
            t0 = time.perf_counter()
            O.dequant_index_k(m["kv_cache"].numpy().reshape(4096, -1), m["token_loc"].numpy())
            dt, nn = time.perf_counter() - t0, n
        rec["cpu_baseline"] = {"value": nn * per_tok / dt / 1e9, "unit": "GB/s", "cores": _threads(), "kind": "port",
                               "sample": f"{nn} tokens, oracle dequant ({dt:.2f} s)"}
    del np
    return rec


def sec_kstore(args, local):
    """Indexer-K cache writer: 131072 bf16 K rows quantised into permuted slots of a 4096-page pool."""
    import torch

    import hcu_ops

    dev = torch.device("cuda", local)
    n, pool_pages = 131072, 4096
    per_tok = 256 + 4 + 132
    inst = []
    for i in range(_instances(n * per_tok + pool_pages * 64 * 132)):
        g = torch.Generator(device=dev)
        g.manual_seed(i)
        k = torch.randn(n, 128, generator=g, device=dev).to(torch.bfloat16)
        loc = torch.randperm(pool_pages * 64, generator=g, device=dev)[:n].to(torch.int32)
        inst.append((k, loc, torch.zeros(pool_pages, 64, 1, 132, dtype=torch.uint8, device=dev)))
    fns = [lambda m=m: hcu_ops.quant_store_index_k(*m) for m in inst]
    alg = per_tok * n
    ms, clocks, launches = _hbm_loop(fns, alg, args.steps, local, dev)
    gbs = alg / (ms * 1e-3) / 1e9
    hbm, _, src = _peaks()
    rec = _rec("indexer-K cache writer throughput (algorithmic bytes / s)", gbs, "GB/s", ms, launches,
               f"indexer-K writer: {n} bf16 rows -> fp8 + scale into permuted slots of {pool_pages} pages; "
               f"graph-replayed launches cycling {len(fns)} sets", tokens=n, bytes_per_token=per_tok)
    rec["dtype"] = "bf16 -> fp32 -> fp8e4m3"
    rec["roofline"] = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                       "traffic": _profile_traffic("quant_store_index_k_kernel"), "kernel": "quant_store_index_k_kernel",
                       "alg_bytes_per_launch": alg, "peak_source": src}
    rec["gpu_launches"] = launches
    rec["clocks"] = clocks
    if not args.no_cpu_baseline:
        import numpy as np

        from oracle import indexer as O

        g = torch.Generator().manual_seed(0)
        kc = torch.randn(n, 128, generator=g).to(torch.bfloat16).float().numpy()
        locc = torch.randperm(pool_pages * 64, generator=g)[:n].to(torch.int32).numpy()
        pool = np.zeros((pool_pages, 64 * 132), np.uint8)
        t0 = time.perf_counter()
        O.quant_store_index_k(kc, locc, pool)
        dt = time.perf_counter() - t0
        rec["cpu_baseline"] = {"value": n * per_tok / dt / 1e9, "unit": "GB/s", "cores": _threads(), "kind": "port",
                               "sample": f"{n} tokens (whole workload), oracle writer ({dt:.2f} s)"}
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


def sec_mla_kv(args, local):
    """MLA decode front end (rope_qout_kv_store): 128 tokens x 64 q heads per call, q rotated in place."""
    import numpy as np
    import torch

    import hcu_ops

    dev = torch.device("cuda", local)
    packed, q, pos, cache, w, loc, buf = _mla_inputs(dev, MLA_T, 0)
    kv_c, k_pe, q_pe = packed[:, 2048:2560], packed[:, 2560:].unsqueeze(1), q[..., 192:]
    fn = lambda: hcu_ops.rope_qout_kv_store(pos, q_pe, q_pe, kv_c, w, 1e-6, k_pe, cache, False, buf, loc)  # noqa
    for _ in range(5):
        fn()
    iters = max(10, min(args.steps, 200))
    ms, clocks = _per_launch(fn, iters, _read_flush(dev), local)
    alg = MLA_BYTES_PER_TOKEN * MLA_T + 1024
    gbs = alg / (ms * 1e-3) / 1e9
    hbm, _, src = _peaks()
    rec = _rec("MLA decode front end latency (us per call, 128 tokens x 64 q heads)", ms * 1e3, "us", ms, iters,
               "MLA front end: q rope (64 heads), latent RMS norm in place, k rope, fp8 656-byte slot store, 128 "
               "decode tokens; L2 flushed (read) before every call", higher=False, tokens=MLA_T,
               bytes_per_token=MLA_BYTES_PER_TOKEN)
    rec["dtype"] = "bf16 -> fp32 -> bf16 / fp8e4m3"
    rec["roofline"] = {"bound": "latency", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                       "traffic": None, "alg_bytes_per_launch": alg, "peak_source": src,
                       "note": "2.5 MB per call: latency-bound, roofline not claimed"}
    rec["gpu_launches"] = iters
    rec["clocks"] = clocks
    if not args.no_cpu_baseline:
        from oracle import mla as M

        packed, q, pos, cache, w, loc, buf = _mla_inputs(torch.device("cpu"), MLA_T, 0)
        u = lambda x: x.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        t0 = time.perf_counter()
        M.rope_qout_kv_store(pos.numpy(), u(q[..., 192:]), u(packed[:, 2048:2560]), u(w), 1e-6, u(packed[:, 2560:]),
                             u(cache), False, buf.numpy(), loc.numpy())
        dt = time.perf_counter() - t0
        rec["cpu_baseline"] = {"value": dt * 1e6, "unit": "us", "cores": _threads(), "kind": "port",
                               "sample": f"one call, {MLA_T} tokens x {MLA_H} q heads (whole workload)"}
    return rec


def sec_cp_filter(args, local):
    """One rank's share of config 4's bounded exchange at P = 8 (rank 3 of 8, balanced ranges): the sampled
    per-row bound and the filter over that rank's materialised local logits (16384 rows x its range),
    timed over the rank's real logits; HBM-bound reads of the logits and mask."""
    import torch

    import hcu_ops
    from hcu_ops.cp import kv_range, list_len, local_rows

    dev = torch.device("cuda", local)
    rows, N, P, r = CP_ROWS, CP_N, 8, 3
    w = _workloads().make_ragged(rows, N - rows, heads=64, seed=0, device=dev)
    lo, hi = kv_range(r, P, N, causal_rows=rows)
    lens = local_rows(w["row_end"], lo, hi)
    lg, mk = hcu_ops.mqa_logits_ragged(w["q"], w["k_fp8"][lo:hi].contiguous(), w["k_scale"][lo:hi].contiguous(),
                                       w["weights"], torch.zeros_like(lens), lens)
    del w["k_fp8"]
    vis = (w["row_end"].clamp(max=N)).to(torch.int32)
    gtab = (torch.arange(hi - lo, dtype=torch.int32, device=dev) + lo).expand(rows, hi - lo)
    cap = list_len(P)
    send = torch.empty((P, 2, rows // P, cap), dtype=torch.int32, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    state = {}

    def bound():
        state["b"] = hcu_ops.cp_local_bound(lg, mk, lens, vis)

    def filt():
        hcu_ops.cp_filter(lg, mk, lens, gtab, state["b"], send, flag)

    for _ in range(3):
        bound()
        filt()
    iters = max(3, min(args.steps, 20))
    ms_b, _ = _timed(bound, iters, local)
    ms, clocks = _timed(filt, iters, local)
    width = hi - lo
    nbytes = rows * width * 4 + rows * (width // 16) * 2 + send.numel() * 4
    hbm, _, src = _peaks()
    rec = _rec("CP bounded-exchange filter throughput, one rank at P = 8 (algorithmic bytes / s)",
               nbytes / (ms * 1e-3) / 1e9, "GB/s", ms, iters,
               f"config4 rank {r} of {P}: {rows} rows x {width} local tokens (materialised logits "
               f"{rows * width * 4 / 1e9:.2f} GB > L2), {cap}-slot lists; bound timed separately", rows=rows,
               width=width)
    rec["bound_ms"] = ms_b
    rec["flag"] = int(flag.item())
    rec["roofline"] = {"bound": "hbm", "achieved": nbytes / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                       "frac": nbytes / (ms * 1e-3) / 1e9 / hbm, "traffic": None, "kernel": "cp_filter_kernel<512>",
                       "alg_bytes_per_launch": nbytes, "peak_source": src}
    rec["gpu_launches"] = iters * 2
    rec["clocks"] = clocks
    if not args.no_cpu_baseline:
        from oracle import indexer as O

        sel = _stratified(rows, 2048)
        sl = torch.as_tensor(sel, device=dev)
        x, m = lg[sl].cpu().numpy(), mk[sl].cpu().numpy()
        ln, bb, gt = lens[sl].cpu().numpy(), state["b"][sl].cpu().numpy(), gtab[sl].cpu().numpy()
        t0 = time.perf_counter()
        O.cp_filter(x, m, ln, gt, bb, cap)
        dt = time.perf_counter() - t0
        cb = len(sel) * (width * 4 + (width // 16) * 2 + 2 * cap * 4)
        rec["cpu_baseline"] = {"value": cb / dt / 1e9, "unit": "GB/s", "cores": _threads(), "kind": "port",
                               "sample": f"{len(sel)} stratified rows of {rows} through the oracle's filter ({dt:.2f} s)"}
    return rec


SECONDARY = {"decode0": sec_decode0, "prefill": sec_prefill, "dequant": sec_dequant,
             "mla_dequant": lambda a, l: sec_dequant(a, l, mla=True), "kstore": sec_kstore, "mla_kv": sec_mla_kv,
             "cp_filter": sec_cp_filter}


def _standalone(args, world, rank, local):
    """--workload NAME: one secondary workload (or config 4) as its own JSON line."""
    if args.workload == "cp_prefill":
        rec = run_cp_prefill(args, world, rank, local)
    elif rank == 0:
        rec = SECONDARY[args.workload](args, local)
    else:
        rec = None
    if rec is not None:
        rec.update({"n_gpus": world, "warmup": args.warmup, "vs_baseline": None,
                    "data": "synthetic (seeded)", "dtype": rec.get("dtype", DTYPE)})
        rec.setdefault("scaling", "weak")
    return rec


def run_reference_sample(args):
    """--impl reference --workload NAME: the CPU oracle on a bounded sample of that workload."""
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    wl = args.workload
    if wl in ("prefill", "cp_prefill"):
        rows, prefix = (8192, 65536) if wl == "prefill" else (CP_ROWS, CP_N - CP_ROWS)
        v, sample = _ragged_cpu_sample(rows, prefix)
        unit = "G-scores/s"
    else:
        a = argparse.Namespace(**vars(args))
        a.no_cpu_baseline = False
        rec = None
        import torch as _t

        if not _t.cuda.is_available():
            raise SystemExit("--impl reference --workload " + wl + ": that sample reuses the GPU workload's setup")
        rec = SECONDARY[wl](a, 0)
        v, unit, sample = rec["cpu_baseline"]["value"], rec["cpu_baseline"]["unit"], rec["cpu_baseline"]["sample"]
    return {"impl": "reference", "metric": f"{wl} (CPU oracle)", "value": v, "unit": unit, "n_gpus": 0,
            "steps": 1, "warmup": 0, "higher_is_better": unit != "us", "config": {"workload": wl},
            "cpu_baseline": {"value": v, "unit": unit, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="headline and cp_prefill only")
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
            cp = run_cp_prefill(args, world, rank, local)
            if rank == 0:
                rec["cp_prefill"] = cp
                if world == 1 and not args.no_secondary:
                    sec = {}
                    for name, fn in SECONDARY.items():
                        sec[name] = fn(args, local)
                        torch.cuda.empty_cache()
                    rec["secondary"] = sec
        elif args.workload in SECONDARY or args.workload == "cp_prefill":
            rec = _standalone(args, world, rank, local)
        else:
            raise SystemExit(f"unknown workload {args.workload}")
        if rec is not None:
            print(json.dumps(rec), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
