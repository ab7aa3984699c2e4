"""Seeded synthetic inputs with the shapes and value distributions of the indexer configs.

The reference measures on live GLM-5.3 serving traffic; these generators stand in
for it: q ~ N(0,1) quantised per row to fp8 e4m3 with an amax/448 fp32 scale
(folded into the head weights, as the indexer's caller does), K ~ N(0,1)
quantised per token the same way and stored in 64-token pages laid out as the
logits op reads them (``[page][64 x 128 fp8 | 64 x fp32 scale]``,
``hcu_ops/csrc/mqa_hist.cu:77-91`` of the reference), head weights ~ N(0,1)/8.

Everything is generated with a seeded ``torch.Generator`` on the requested
device; CPU and GPU streams differ, so tests that compare against the CPU
oracle generate on the CPU and copy to the device.
"""
from __future__ import annotations

import math

import torch

PAGE = 64
HEAD_DIM = 128
PAGE_BYTES = PAGE * (HEAD_DIM + 4)  # 8448
FP8_MAX = 448.0


def quant_rows_fp8(x: torch.Tensor):
    """Per-row amax/448 fp8 e4m3 quantisation -> (fp8 tensor, fp32 scale [rows])."""
    amax = x.abs().amax(-1).clamp_min(1e-12)
    scale = (amax / FP8_MAX).float()
    q = (x / scale[..., None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q, scale


def pack_index_k_pages(k_fp8: torch.Tensor, k_scale: torch.Tensor) -> torch.Tensor:
    """Token-major fp8 K ``[n_pages*64, 128]`` + scales -> pages ``[n_pages, 64, 1, 132]`` uint8."""
    n_pages = k_fp8.shape[0] // PAGE
    fp8 = k_fp8.view(torch.uint8).reshape(n_pages, PAGE * HEAD_DIM)
    sc = k_scale.float().contiguous().view(torch.uint8).reshape(n_pages, PAGE * 4)
    return torch.cat([fp8, sc], 1).contiguous().view(n_pages, PAGE, 1, HEAD_DIM + 4)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_decode(batch_reqs: int, next_n: int, ctx_lens, heads: int = 64, seed: int = 0,
                device="cpu", width_pages: int | None = None, extra_pages: int = 0):
    """Decode indexer inputs (configs 0 and 1).

    ``ctx_lens``: per-request context lengths ``L_r``; row ``j`` of request
    ``r`` sees ``L_r - next_n + 1 + j`` tokens (the last row sees ``L_r``).
    Pages of all requests live in one shuffled pool; the block table of every
    row of a request holds that request's pages; ``page_table_size_1`` maps a
    token index to its KV slot ``page * 64 + offset``.
    """
    g = _gen(seed, device)
    lens_req = [int(x) for x in ctx_lens]
    pages_req = [(L + PAGE - 1) // PAGE for L in lens_req]
    n_pages = sum(pages_req) + extra_pages
    width_pages = width_pages or max(pages_req)
    B = batch_reqs * next_n
    x = torch.randn(B, heads, HEAD_DIM, generator=g, device=device)
    qf, qs = quant_rows_fp8(x.reshape(B, heads * HEAD_DIM))
    q = qf.view(B, 1, heads, HEAD_DIM)
    w = torch.randn(B, heads, generator=g, device=device) / 8.0
    weights = (w * qs[:, None]).float().contiguous()
    k = torch.randn(n_pages * PAGE, HEAD_DIM, generator=g, device=device)
    kf, ks = quant_rows_fp8(k)
    kv = pack_index_k_pages(kf, ks)
    perm = torch.randperm(n_pages, generator=g, device=device).to(torch.int32)
    bt = torch.zeros(B, width_pages, dtype=torch.int32, device=device)
    lens = torch.empty(B, dtype=torch.int32, device=device)
    off = 0
    for r, (L, P) in enumerate(zip(lens_req, pages_req)):
        rows = slice(r * next_n, (r + 1) * next_n)
        bt[rows, :P] = perm[off:off + P]
        off += P
        lens[rows] = torch.arange(L - next_n + 1, L + 1, dtype=torch.int32, device=device)
    width = width_pages * PAGE
    tok = torch.arange(width, device=device, dtype=torch.int32)
    pt = (bt.long()[:, tok.long() // PAGE] * PAGE + (tok.long() % PAGE)[None, :]).to(torch.int32)
    cu = torch.arange(B + 1, dtype=torch.int32, device=device)
    return dict(q=q, kv_cache=kv, weights=weights, context_lens=lens, block_table=bt,
                max_context_len=width, group_size=next_n, page_table_size_1=pt.contiguous(),
                cu_seqlens_q=cu, heads=heads)


def config0(device="cpu", seed=0):
    """Config 0: 1 request, 1 row, 64 heads, 8192-token context in a permuted pool."""
    return make_decode(1, 1, [8192], heads=64, seed=seed, device=device)


def config1_lens(seed=0, reqs=64, lo=4096, hi=65536):
    g = torch.Generator().manual_seed(seed + 1)
    return torch.randint(lo, hi + 1, (reqs,), generator=g).tolist()


def config1(device="cpu", seed=0, reqs=64, lo=4096, hi=65536):
    """Config 1: 64 requests x next_n=2 rows, contexts U[4096, 65536], shared shuffled pool."""
    return make_decode(reqs, 2, config1_lens(seed, reqs, lo, hi), heads=64, seed=seed,
                       device=device, width_pages=(hi + PAGE - 1) // PAGE)


def make_ragged(rows: int, prefix: int, heads: int = 64, seed: int = 0, device="cpu",
                n_tokens: int | None = None):
    """Prefill chunk (config 2 shape): row i sees tokens ``[0, prefix + i + 1)`` of a contiguous K."""
    g = _gen(seed, device)
    N = n_tokens if n_tokens is not None else prefix + rows
    x = torch.randn(rows, heads * HEAD_DIM, generator=g, device=device)
    qf, qs = quant_rows_fp8(x)
    w = torch.randn(rows, heads, generator=g, device=device) / 8.0
    weights = (w * qs[:, None]).float().contiguous()
    k = torch.randn(N, HEAD_DIM, generator=g, device=device)
    kf, ks = quant_rows_fp8(k)
    ar = torch.arange(rows, device=device, dtype=torch.int32)
    ks_row = torch.zeros(rows, dtype=torch.int32, device=device)
    ke_row = (prefix + ar + 1).to(torch.int32).clamp(max=N)
    return dict(q=qf.view(rows, heads, HEAD_DIM), k_fp8=kf.contiguous(), k_scale=ks.contiguous(),
                weights=weights, row_start=ks_row, row_end=ke_row, heads=heads)


def make_index_k_dequant(n_tokens: int, pool_pages: int, seed: int = 0, device="cpu"):
    """Config 3: ``n_tokens`` tokens over ``n_tokens/64`` randomly chosen, permuted pages of a pool."""
    g = _gen(seed, device)
    k = torch.randn(pool_pages * PAGE, HEAD_DIM, generator=g, device=device)
    kf, ks = quant_rows_fp8(k)
    kv = pack_index_k_pages(kf, ks)
    used = math.ceil(n_tokens / PAGE)
    pages = torch.randperm(pool_pages, generator=g, device=device)[:used].long()
    tok = torch.arange(n_tokens, device=device)
    loc = (pages[tok // PAGE] * PAGE + tok % PAGE).to(torch.int32)
    return dict(kv_cache=kv, token_loc=loc.contiguous())


def make_mla_dequant(n_tokens: int, pool: int, seed: int = 0, device="cpu", exact_scales=False):
    """656-byte MLA slots ``[pool, 1, 656]``: 512 fp8 | 4 fp32 scales | 64 bf16 rope, random slot table.

    ``exact_scales`` draws the scales from fp8-representable values so every
    fp32 product is exact in bf16 (used to pin layouts independently of rounding).
    """
    g = _gen(seed, device)
    nope = (torch.randn(pool, 512, generator=g, device=device)).to(torch.float8_e4m3fn).view(torch.uint8)
    if exact_scales:
        s = (torch.rand(pool, 4, generator=g, device=device) * 0.05 + 0.002).to(torch.float8_e4m3fn).float()
    else:
        s = torch.rand(pool, 4, generator=g, device=device) * 0.05 + 0.002
    rope = torch.randn(pool, 64, generator=g, device=device).to(torch.bfloat16)
    cache = torch.cat([nope, s.float().contiguous().view(torch.uint8),
                       rope.contiguous().view(torch.uint8)], 1).contiguous().view(pool, 1, 656)
    page = torch.randint(0, pool, (n_tokens,), generator=g, device=device, dtype=torch.int32)
    return dict(quant_k_cache=cache, page_table_1_flattened=page)
