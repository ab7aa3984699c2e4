"""Generate the golden fixtures of tests/golden/ by executing the reference's own code on CPU.

Run once in a container that has the reference checkout (it is not needed at
test time and does not exist on the GPU machines):

    python tests/golden/make_golden.py /path/to/reference

What is executed from the reference (extracted with ``ast`` from the files, so
their module-level GPU / lightop code does not run):
  * ``make`` of ``hcu_ops/tests/topk_lib.py:8-51`` -- the reference's ten score
    distributions with NaN-poisoned unset slots, ragged lengths and the
    ``arange + 7 + 1e6*row`` page table; run with ``dev = "cpu"`` after
    ``torch.manual_seed(0)``;
  * ``same_values`` of ``topk_lib.py:70-89`` -- the reference's top-k validity
    criterion, applied here to an independent ``torch.topk`` selection to
    confirm the stored expected value multisets;
  * ``mask_bits`` / ``ref_hist`` of ``hcu_ops/tests/test_mqa_hist.py:105-124``
    -- the pass-1 histogram + (positives, zeros) reference;
  * the Triton kernel ``_dequantize_k_cache_paged_v2_kernel`` and its host
    wrapper ``dequantize_k_cache_paged`` of
    ``prefill/patches/patch_fast_dequant.py:36-98``, under
    ``TRITON_INTERPRET=1``.  The interpreter truncates fp32 -> bf16 where GPU
    Triton rounds to nearest-even, so the scales are drawn from
    fp8-representable values: every product then has at most 8 significant bits
    and is exact in bf16, which makes the interpreter's output the exact answer
    and pins the slot layout, group/scale mapping and rope copy bit for bit.

Outputs: topk_make_cases.npz, ref_hist_cases.npz, dequant_mla_triton.npz.
"""
from __future__ import annotations

import ast
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def load_functions(path, names, extra_globals):
    src = open(path, encoding="utf-8").read()
    tree = ast.parse(src)
    ns = dict(extra_globals)
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            code = ast.get_source_segment(src, node)
            exec(compile(code, path, "exec"), ns)  # noqa: S102 -- reference test helper
    missing = [n for n in names if n not in ns]
    assert not missing, f"{path}: missing {missing}"
    return ns


def topk_cases(ref):
    ns = load_functions(os.path.join(ref, "hcu_ops/tests/topk_lib.py"), ["make", "same_values"],
                        {"torch": torch, "dev": "cpu"})
    make, same_values = ns["make"], ns["same_values"]
    torch.manual_seed(0)
    cases = {}
    dists = ["pos", "sparse30", "sparse2", "relu_sum", "mixed", "ties", "zeros", "neg", "narrow", "const"]
    n = 0
    for dist in dists:
        for L in (1000, 2049, 4096):
            if L == 1000 and dist not in ("relu_sum", "neg"):
                continue
            for ragged in (False, True):
                B = 2
                W = L + 64
                x, mask, lengths, pt, cu = make(B, L, dist, W=W, ragged=ragged)
                # expected: the top-2048 value multiset (unset -> 0, pads -> -inf), validated with
                # the reference's own criterion against an independent torch.topk selection
                xv = torch.nan_to_num(x, nan=0.0)
                ref = torch.full((B, 2048), -1, dtype=torch.int32)
                for b in range(B):
                    Lb = int(min(lengths[b], W))
                    k = min(Lb, 2048)
                    idx = torch.topk(xv[b, :Lb], k).indices if Lb > 2048 else torch.arange(Lb)
                    ref[b, :k] = pt[b, idx]
                assert same_values(x, lengths, ref, ref)
                vals = torch.where(ref >= 0, torch.gather(xv, 1, (ref - pt[:, :1]).long().clamp(min=0)),
                                   torch.full(ref.shape, -float("inf"))).sort(-1).values
                key = f"c{n:02d}"
                cases[f"{key}_x"] = x.numpy()
                cases[f"{key}_mask"] = mask.numpy()
                cases[f"{key}_lengths"] = lengths.numpy()
                cases[f"{key}_pt"] = pt.numpy()
                cases[f"{key}_sorted_values"] = vals.numpy()
                cases[f"{key}_meta"] = np.array([dists.index(dist), L, int(ragged), W], np.int32)
                n += 1
    cases["n"] = np.array(n)
    np.savez_compressed(os.path.join(OUT, "topk_make_cases.npz"), **cases)
    return n


def hist_cases(ref):
    width = 6144
    ns = load_functions(os.path.join(ref, "hcu_ops/tests/test_mqa_hist.py"), ["mask_bits", "ref_hist"],
                        {"torch": torch, "dev": "cpu", "WIDTH": width})
    ns["bits16"] = torch.arange(16, dtype=torch.int32)
    mk = load_functions(os.path.join(ref, "hcu_ops/tests/topk_lib.py"), ["make"], {"torch": torch, "dev": "cpu"})
    torch.manual_seed(1)
    out = {}
    n = 0
    for dist in ("relu_sum", "mixed", "sparse2", "neg", "const"):
        B = 4
        x, mask, _, _, _ = mk["make"](B, 5000, dist, W=width)
        lens = torch.tensor([5000, 2048, 2049, 7000], dtype=torch.int32)  # below / at / above 2048, > width
        mm = ns["mask_bits"](mask, width)
        g1, cnt = ns["ref_hist"](x, mm, lens)
        out[f"h{n}_x"] = x.numpy()
        out[f"h{n}_mask"] = mask.numpy()
        out[f"h{n}_lens"] = lens.numpy()
        out[f"h{n}_g1"] = g1.numpy().astype(np.int32)
        out[f"h{n}_cnt"] = cnt.numpy().astype(np.int32)
        n += 1
    out["n"] = np.array(n)
    out["width"] = np.array(width)
    np.savez_compressed(os.path.join(OUT, "ref_hist_cases.npz"), **out)
    return n


def dequant_case(ref):
    import triton
    import triton.language as tl

    path = os.path.join(ref, "prefill/patches/patch_fast_dequant.py")
    tree = ast.parse(open(path, encoding="utf-8").read())
    addition = None
    for node in tree.body:
        if isinstance(node, ast.Assign) and getattr(node.targets[0], "id", "") == "ADDITION":
            addition = node.value.value
    assert addition is not None
    sub = ast.parse(addition)
    lines = addition.splitlines()
    parts = ["import torch", "import triton", "import triton.language as tl",
             "_FD_ON = True", "_FD_T = 8", "_FD_WARPS = 4", "_dequantize_k_cache_paged_orig = None"]
    for node in sub.body:
        if isinstance(node, ast.FunctionDef) and node.name in ("_dequantize_k_cache_paged_v2_kernel",
                                                               "dequantize_k_cache_paged"):
            first = min([d.lineno for d in node.decorator_list] + [node.lineno])
            parts.append("\n".join(lines[first - 1:node.end_lineno]))
    # triton.jit reads the kernel's source text, so the extracted code becomes a real module
    import importlib.util
    import tempfile
    tmp = tempfile.NamedTemporaryFile("w", suffix="_ref_dequant.py", delete=False)
    tmp.write("\n\n".join(parts) + "\n")
    tmp.close()
    spec = importlib.util.spec_from_file_location("ref_dequant_v2", tmp.name)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    ns = vars(mod)
    g = torch.Generator().manual_seed(3)
    pool, n = 40, 29  # n not a multiple of the kernel's 8 tokens per program
    nope = torch.randn(pool, 512, generator=g).to(torch.float8_e4m3fn).view(torch.uint8)
    scales = (torch.rand(pool, 4, generator=g) * 0.05 + 0.002).to(torch.float8_e4m3fn).float()
    rope = torch.randn(pool, 64, generator=g).to(torch.bfloat16)
    cache = torch.cat([nope, scales.contiguous().view(torch.uint8), rope.contiguous().view(torch.uint8)], 1)
    cache = cache.contiguous().view(torch.float8_e4m3fn).view(pool, 1, 656)
    page = torch.randint(0, pool, (n,), generator=g, dtype=torch.int32)
    out = ns["dequantize_k_cache_paged"](cache, page)
    np.savez_compressed(os.path.join(OUT, "dequant_mla_triton.npz"), cache=cache.view(torch.uint8).numpy(),
                        page=page.numpy(), out_bits=out.view(torch.int16).numpy())
    return n


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python make_golden.py <path of the reference checkout>")
    ref = sys.argv[1]
    print("topk cases", topk_cases(ref))
    print("hist cases", hist_cases(ref))
    print("dequant tokens", dequant_case(ref))
