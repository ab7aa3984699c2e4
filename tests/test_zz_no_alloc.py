"""The allocation-free top-k entry point, called through the C ABI.

Some callers cannot allocate device memory: code running inside a serving engine that owns the
device's memory pool, or a plug-in invoked where a cudaMalloc would synchronise the device or break
its memory budget.  `hcu_sparse_mask_topk_transform_noalloc` serves them: it keeps its workspace in a
fixed device array of the library instead of asking for one.  These checks compare it with the
regular entry point `hcu_sparse_mask_topk_transform` (exact: same selection, same order) on two calls
in a row -- the second with other shapes and values, so a workspace left over from the first call
would show -- and check that a batch beyond the fixed maximum is refused with an error message.

The file is named so that pytest collects it last."""
import ctypes

import pytest
import torch

from indexer_testlib import make_scores

pytestmark = pytest.mark.gpu

HCU_OK, HCU_ERR_ARG = 0, 1
_ARGS = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]


@pytest.fixture(scope="module")
def lib(hcu):
    so = ctypes.CDLL(hcu.library_path())
    for name in ("hcu_sparse_mask_topk_transform", "hcu_sparse_mask_topk_transform_noalloc"):
        fn = getattr(so, name)
        fn.restype = ctypes.c_int
        fn.argtypes = _ARGS
    so.hcu_topk_noalloc_max_rows.restype = ctypes.c_int64
    so.hcu_last_error_string.restype = ctypes.c_char_p
    return so


def _call(fn, x, mask, lens, pt, out, width=None):
    stream = torch.cuda.current_stream().cuda_stream
    width = x.shape[1] if width is None else width
    return fn(x.data_ptr(), x.shape[0], width, x.stride(0), mask.data_ptr(), mask.stride(0), lens.data_ptr(),
              pt.data_ptr(), pt.stride(0), 2048, out.data_ptr(), stream)


def test_noalloc_topk_equals_regular_entry_point_twice(lib, dev):
    max_rows = lib.hcu_topk_noalloc_max_rows()
    assert max_rows >= 128
    # two calls in a row with different batches: wide rows, then narrower rows of another distribution
    for rows, L, W, dist, seed in [(max_rows, 40000, 40064, "relu_sum", 1), (37, 9000, 9216, "ties", 2)]:
        x, mask, lens, pt = make_scores(rows, L, dist, W=W, ragged=True, seed=seed)
        x, mask, lens, pt = (t.to(dev) for t in (x, mask, lens, pt))
        ref = torch.full((rows, 2048), -7, dtype=torch.int32, device=dev)
        got = torch.full((rows, 2048), -9, dtype=torch.int32, device=dev)
        assert _call(lib.hcu_sparse_mask_topk_transform, x, mask, lens, pt, ref) == HCU_OK
        assert _call(lib.hcu_sparse_mask_topk_transform_noalloc, x, mask, lens, pt, got) == HCU_OK
        torch.cuda.synchronize()
        assert torch.equal(got, ref), (rows, dist)


def _edge_case(kind, dev):
    """Scores whose rows take the entry point's edge paths: an empty width (nothing to select, every
    output -1), widths of at most 2048 (every row short: its page-table entries in order), and a score
    row stride that is not a multiple of 4 floats (the scalar-load kernel instance)."""
    g = torch.Generator().manual_seed(5)
    if kind == "width0":
        rows, W = 7, 0
        x = torch.rand(rows, 16, generator=g)
        mask = torch.zeros(rows, 1, dtype=torch.int16)
        lens = torch.tensor([0, 5, 100, 0, 3000, 1, 2], dtype=torch.int32)
    elif kind == "short":
        rows, W = 19, 2048
        x = torch.rand(rows, W, generator=g)
        mask = torch.full((rows, W // 16), -1, dtype=torch.int16)
        lens = torch.randint(0, 2100, (rows,), generator=g, dtype=torch.int32)
    else:  # "odd_stride"
        rows, W = 23, 12000
        x = torch.rand(rows, W + 3, generator=g)[:, :W]
        mask = torch.full((rows, (W + 15) // 16), -1, dtype=torch.int16)
        lens = torch.randint(1000, W + 1, (rows,), generator=g, dtype=torch.int32)
    pt = torch.randint(0, 1 << 30, (rows, max(W, 16)), generator=g, dtype=torch.int32)
    x, mask, lens, pt = (t.to(dev) for t in (x, mask, lens, pt))
    # width0: the rows of a real allocation (non-null pointer, row stride 16) passed with width 0
    return x, mask, lens, pt, W


@pytest.mark.parametrize("kind", ["width0", "short", "odd_stride"])
def test_noalloc_topk_edge_shapes_twice(lib, dev, kind):
    x, mask, lens, pt, W = _edge_case(kind, dev)
    rows = x.shape[0]
    for _ in range(2):  # the second call sees whatever the first left in the fixed array
        ref = torch.full((rows, 2048), -7, dtype=torch.int32, device=dev)
        got = torch.full((rows, 2048), -9, dtype=torch.int32, device=dev)
        assert _call(lib.hcu_sparse_mask_topk_transform, x, mask, lens, pt, ref, W) == HCU_OK
        assert _call(lib.hcu_sparse_mask_topk_transform_noalloc, x, mask, lens, pt, got, W) == HCU_OK
        torch.cuda.synchronize()
        assert torch.equal(got, ref), kind
    if kind == "width0":
        assert (got == -1).all()


def test_noalloc_topk_refuses_rows_beyond_its_maximum(lib, dev):
    rows = lib.hcu_topk_noalloc_max_rows() + 1
    x, mask, lens, pt = make_scores(rows, 4096, "pos", seed=3)
    x, mask, lens, pt = (t.to(dev) for t in (x, mask, lens, pt))
    out = torch.full((rows, 2048), -5, dtype=torch.int32, device=dev)
    assert _call(lib.hcu_sparse_mask_topk_transform_noalloc, x, mask, lens, pt, out) == HCU_ERR_ARG
    assert b"maximum" in lib.hcu_last_error_string()
    torch.cuda.synchronize()
    assert (out == -5).all()  # nothing was launched
