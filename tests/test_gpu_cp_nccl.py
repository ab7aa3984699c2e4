"""Context-parallel prefill on 2 GPUs: every rank's result equals the 1-GPU result.

Each rank scores its own KV range with the ragged logits kernel and the ranks exchange and merge
per-range lists: over peer memory (the default: the kernels store bounds, lists and merged rows
into the other rank's buffers over NVLink and wait for its per-step flags; three steps in a row,
so the step counter advances) or over NCCL -- the bounded lists (an all-reduce MIN of sampled
bounds, then every token at or above the bound) or local top-2048 lists (the exact path),
row-sharded all-to-all then an all-gather of the final indices, and the all-gather mode.  Skipped
with fewer than two visible GPUs.  Ranks are spawned processes with NVLS off and a short
process-group timeout, so a rank that fails ends the others' collectives with an error instead of
a wait; the peer kernels' waits are bounded (2 s)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROWS, PREFIX = 300, 20000


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, mode, q):
    mode, _, variant = mode.partition(":")
    import datetime
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    for p in (os.path.dirname(here), os.path.join(os.path.dirname(here), "sglang0.5.18-opt_b200")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from hcu_ops.cp import cp_prefill_topk, kv_range
        from hcu_ops.workloads import make_ragged

        w = make_ragged(ROWS, PREFIX, heads=64, seed=5)
        N = w["k_fp8"].shape[0]
        cr = ROWS if variant == "balanced" else 0
        lo, hi = kv_range(rank, world, N, causal_rows=cr)
        stats = {}
        outs = []
        for _ in range(3 if mode == "peer" else 1):
            out = cp_prefill_topk(w["q"].to(dev), w["k_fp8"][lo:hi].contiguous().to(dev),
                                  w["k_scale"][lo:hi].contiguous().to(dev), w["weights"].to(dev),
                                  w["row_end"].to(dev), N, mode=mode, bounded=variant != "exact", causal_rows=cr,
                                  stats=stats)
            outs.append(out.clone())
        torch.cuda.synchronize()
        from hcu_ops import read_device_status

        q.put((rank, [o.cpu().numpy() for o in outs], stats.get("exchange", ""), read_device_status(clear=True)))
    except Exception as e:  # reported to the parent; the process group timeout ends the peer
        q.put((rank, repr(e), "", 0))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["peer", "peer:balanced", "rowshard", "rowshard:exact", "rowshard:balanced",
                                  "allgather"])
def test_cp_nccl_two_gpus_equals_one_gpu(hcu, dev, mode):
    from hcu_ops.cp import cp_prefill_topk
    from hcu_ops.workloads import make_ragged

    w = make_ragged(ROWS, PREFIX, heads=64, seed=5)
    N = w["k_fp8"].shape[0]
    ref = cp_prefill_topk(w["q"].to(dev), w["k_fp8"].to(dev), w["k_scale"].to(dev), w["weights"].to(dev),
                          w["row_end"].to(dev), N).cpu().numpy()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            r, outs, exchange, status = q.get(timeout=300)
            got[r] = (outs, exchange, status)
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    for r in range(2):
        outs, exchange, status = got[r]
        assert isinstance(outs, list), outs
        assert status == 0, f"rank {r}: device status {status:#x}"
        if mode.startswith("peer"):
            assert exchange.startswith("peer memory"), exchange
        for i, o in enumerate(outs):
            assert np.array_equal(o, ref), f"rank {r} step {i}: {(o != ref).sum()} differing entries"
