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
