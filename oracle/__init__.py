"""CPU oracle for the DSA lightning-indexer path (TEST INFRASTRUCTURE ONLY).

This package restates, on the CPU, what the reference's indexer ops compute:
paged fp8 K-cache dequant, the MQA index logits with their nonzero mask and the
fused top-k pass-1 histogram, the exact causal top-2048 with its page-table
transform, and the context-parallel merge of per-range top-k lists.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import it, and only as the checker or as the timed CPU
baseline. The product path (``hcu_ops``) never imports it and fails loudly
when its CUDA library is missing.

Pinning status (how far the restatement is checked against the reference):
  * dequant: pinned bit-exactly against the reference's own Triton kernel
    (``prefill/patches/patch_fast_dequant.py``) executed in the Triton CPU
    interpreter on inputs whose products are exact in bf16; the rounding step
    (one round-to-nearest-even fp32->bf16) is restated from the same source.
  * pass-1 histogram: pinned against the reference's torch ``ref_hist``
    (``hcu_ops/tests/test_mqa_hist.py:109-124``) executed on CPU.
  * top-k: checked with the reference's own validity criteria (``same_values``
    in ``hcu_ops/tests/topk_lib.py:70-89``, ``topk_values`` in
    ``test_mqa_hist.py:131-144``) on the reference's own score generator
    (``topk_lib.py:8-51``); the bit-exact oracle the reference used (lightop)
    is closed and absent, so the tie order is restated from
    ``hcu_ops/csrc/sparse_mask_topk.cu:1-7,299-348``.
  * logits: restated from ``hcu_ops/csrc/mqa_hist.cu:97-273``; no runnable
    reference exists (HIP for gfx938 + closed lightop), so this stage is
    "parity unpinned" beyond the restatement.
"""
