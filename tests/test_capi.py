"""CPU checks of the C ABI: the library loads, exports every symbol the header declares, and
rejects bad arguments before launching anything (no GPU needed)."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "hcu_indexer.h")
LIB = os.path.join(REPO, "sglang0.5.18-opt_b200", "hcu_ops", "libhcu_indexer.so")

HCU_OK, HCU_ERR_ARG, HCU_ERR_UNSUPPORTED = 0, 1, 4


def declared_symbols():
    text = open(HEADER).read()
    return re.findall(r"^(?:const char\*|int64_t|int)\s+(hcu_\w+)\(", text, re.M)


@pytest.fixture(scope="module")
def lib():
    return ctypes.CDLL(LIB)


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert len(names) >= 14
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_version(lib):
    lib.hcu_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.hcu_version()


def test_workspace_queries(lib):
    lib.hcu_topk_hist_ws_elems.restype = ctypes.c_int64
    lib.hcu_topk_hist_ws_elems.argtypes = [ctypes.c_int64]
    assert lib.hcu_topk_hist_ws_elems(3) == 3 * (2 * 4096 + 2)
    lib.hcu_topk_workspace_bytes.restype = ctypes.c_int64
    lib.hcu_topk_workspace_bytes.argtypes = [ctypes.c_int64] * 3
    assert lib.hcu_topk_workspace_bytes(4, 65536, 8) >= 0


def _topk_args(topk=2048, rows=1, width=4096):
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails or rows == 0 first
    return [p, ctypes.c_int64(rows), ctypes.c_int64(width), ctypes.c_int64(width), p,
            ctypes.c_int64((width + 15) // 16), p, p, ctypes.c_int64(width), ctypes.c_int64(topk), p, None]


def test_topk_rejects_bad_topk_and_accepts_empty(lib):
    f = lib.hcu_sparse_mask_topk_transform
    f.restype = ctypes.c_int
    assert f(*_topk_args(topk=100)) == HCU_ERR_ARG
    assert f(*_topk_args(rows=0)) == HCU_OK
    a = _topk_args()
    a[0] = None  # null score
    assert f(*a) == HCU_ERR_ARG


def test_logits_rejects_unsupported_heads_and_bad_shapes(lib):
    f = lib.hcu_mqa_logits_hist
    f.restype = ctypes.c_int
    p = ctypes.c_void_p(16)
    i64 = ctypes.c_int64

    def call(heads=64, batch=2, G=1, maxctx=4096, page_stride=8448):
        return f(p, i64(batch), i64(heads), p, i64(100), i64(page_stride), p, p, p, i64(maxctx // 64), i64(maxctx),
                 i64(G), i64(0), i64(0), None, p, p, None, None)

    assert call(heads=48) == HCU_ERR_UNSUPPORTED
    assert call(batch=3, G=2) == HCU_ERR_ARG
    assert call(maxctx=100) == HCU_ERR_ARG
    assert call(page_stride=8440) == HCU_ERR_ARG


def test_dequant_rejects_unaligned_stride(lib):
    f = lib.hcu_dequant_k_cache_paged
    f.restype = ctypes.c_int
    p = ctypes.c_void_p(16)
    assert f(p, ctypes.c_int64(10), ctypes.c_int64(650), p, ctypes.c_int64(4), p, None) == HCU_ERR_ARG
    assert f(p, ctypes.c_int64(10), ctypes.c_int64(656), p, ctypes.c_int64(0), p, None) == HCU_OK


def test_merge_rejects_too_many_parts(lib):
    f = lib.hcu_cp_topk_merge
    f.restype = ctypes.c_int
    p = ctypes.c_void_p(16)
    assert f(p, p, ctypes.c_int64(17), ctypes.c_int64(4), p, p, None) == HCU_ERR_ARG
    assert f(p, p, ctypes.c_int64(2), ctypes.c_int64(0), p, p, None) == HCU_OK


def test_cp_bounded_exchange_argument_checks(lib):
    """The bounded-exchange entry points refuse bad shapes before launching anything."""
    p = ctypes.c_void_p(16)
    i64 = ctypes.c_int64
    m = lib.hcu_cp_topk_merge_lists
    m.restype = ctypes.c_int
    # list length not a power of two / too short for 2048 entries / past 2048
    assert m(p, p, i64(2), i64(1000), i64(4000), i64(2), p, None, ctypes.c_int32(1), p, None) == HCU_ERR_ARG
    assert m(p, p, i64(2), i64(512), i64(1024), i64(2), p, None, ctypes.c_int32(1), p, None) == HCU_ERR_ARG
    assert m(p, p, i64(2), i64(4096), i64(8192), i64(2), p, None, ctypes.c_int32(1), p, None) == HCU_ERR_ARG
    assert m(p, p, i64(2), i64(2048), i64(100), i64(2), p, None, ctypes.c_int32(1), p, None) == HCU_ERR_ARG  # part stride
    assert m(p, p, i64(2), i64(2048), i64(4096), i64(0), p, None, ctypes.c_int32(1), p, None) == HCU_OK  # no rows
    f = lib.hcu_cp_filter
    f.restype = ctypes.c_int
    # cap past 2048, and a row block smaller than its lists
    assert f(p, i64(4), i64(64), i64(64), p, i64(4), p, p, i64(0), p, i64(4096), p, p, i64(4), i64(0), None, p,
             None) == HCU_ERR_ARG
    assert f(p, i64(4), i64(64), i64(64), p, i64(4), p, p, i64(0), p, i64(2048), p, p, i64(2), i64(100), None, p,
             None) == HCU_ERR_ARG
    b = lib.hcu_cp_local_bound
    b.restype = ctypes.c_int
    assert b(p, i64(4), i64(64), i64(32), p, i64(4), p, p, p, None) == HCU_ERR_ARG  # stride below width
    assert b(p, i64(0), i64(64), i64(64), p, i64(4), p, p, p, None) == HCU_OK


def test_rope_qout_kv_store_argument_checks(lib):
    """The MLA front end refuses bad arguments before launching anything."""
    f = lib.hcu_rope_qout_kv_store
    f.restype = ctypes.c_int
    p, i64, i32 = ctypes.c_void_p(16), ctypes.c_int64, ctypes.c_int32
    flt = ctypes.c_float

    def call(T=4, kv_tok=512, mode=2, n_loc=4, slot_stride=656):
        return f(p, i32(1), i64(T), p, i64(64), i64(64 * 64), i64(64), p, i64(64 * 64), i64(64), p, i64(kv_tok), p,
                 flt(1e-6), p, i64(64), p, i64(100), i32(0), p, i64(8), i64(slot_stride), p, i64(n_loc), flt(1e-6),
                 i32(mode), None)

    assert call(mode=3) == HCU_ERR_ARG           # no such rsqrt form
    assert call(kv_tok=500) == HCU_ERR_ARG       # latent rows shorter than 512 / not 16-byte multiples
    assert call(n_loc=5) == HCU_ERR_ARG          # more slots than tokens
    assert call(slot_stride=648) == HCU_ERR_ARG  # slots shorter than 656 bytes
    assert call(T=0, n_loc=0) == HCU_OK          # nothing to do


class CpPeers(ctypes.Structure):
    """hcu_cp_peers_t (HCU_CP_MAX_PARTS = 16)."""
    _fields_ = [("parts", ctypes.c_int32), ("rank", ctypes.c_int32), ("rows", ctypes.c_int32),
                ("rows_per_rank", ctypes.c_int32), ("list_len", ctypes.c_int32), ("epoch", ctypes.c_uint32),
                ("ws", ctypes.c_void_p), ("bounds", ctypes.c_void_p * 16), ("lists", ctypes.c_void_p * 16),
                ("lists_exact", ctypes.c_void_p * 16), ("out", ctypes.c_void_p * 16), ("sig", ctypes.c_void_p * 16)]


def test_cp_peer_exchange_argument_checks(lib):
    """The peer-memory exchange refuses a missing or inconsistent description before any launch."""
    fn = lib.hcu_cp_peer_finish
    fn.argtypes = [ctypes.c_int32, ctypes.POINTER(CpPeers), ctypes.c_void_p]
    assert fn(0, None, None) == HCU_ERR_ARG
    fake = 1 << 20  # never dereferenced: every call below is refused by its checks

    def peers(**kw):
        p = CpPeers(parts=2, rank=0, rows=10, rows_per_rank=5, list_len=1024, epoch=1, ws=fake)
        for i in range(2):
            p.bounds[i] = p.lists[i] = p.lists_exact[i] = p.out[i] = p.sig[i] = fake
        for k, v in kw.items():
            setattr(p, k, v)
        return p

    bad = [dict(parts=0), dict(parts=17), dict(rank=2), dict(rows_per_rank=4), dict(list_len=1000),
           dict(list_len=512), dict(epoch=0), dict(ws=None)]
    for b in bad:
        p = peers(**b)
        assert fn(0, ctypes.byref(p), None) == HCU_ERR_ARG, b
    p = peers()
    p.sig[1] = None
    assert fn(0, ctypes.byref(p), None) == HCU_ERR_ARG
    merge = lib.hcu_cp_peer_merge
    merge.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(CpPeers), ctypes.c_void_p]
    assert merge(None, 0, ctypes.byref(peers()), None) == HCU_ERR_ARG  # no totals


def test_wait_limit_entry_point_is_exported(lib):
    lib.hcu_set_wait_limit_ns.argtypes = [ctypes.c_uint64]
    assert hasattr(lib, "hcu_set_wait_limit_ns")


def test_fused_prefill_workspace_and_argument_checks(lib):
    """The fused prefill indexer's workspace query grows with rows and tokens (the exact path's
    logits dominate it), and the entry point refuses bad arguments before launching anything."""
    ws = lib.hcu_mqa_topk_ragged_workspace_bytes
    ws.restype = ctypes.c_int64
    ws.argtypes = [ctypes.c_int64, ctypes.c_int64]
    assert ws(-1, 10) == -1
    small, big = ws(16, 20000), ws(8192, 73728)
    assert 0 < small < big
    assert big >= 8192 * 73728 * 4  # at least the materialised logits of the exact path
    assert ws(8192, 73728) % 256 == 0
    f = lib.hcu_mqa_topk_ragged
    f.restype = ctypes.c_int
    p, i64 = ctypes.c_void_p(16), ctypes.c_int64

    def call(rows=4, heads=64, n=4096, pt_stride=4096, wsb=None, workspace=p):
        b = ws(rows, n) if wsb is None else wsb
        return f(p, i64(rows), i64(heads), p, p, i64(n), p, p, p, i64(pt_stride), p, workspace, i64(b), None, None)

    assert call(heads=48) == HCU_ERR_UNSUPPORTED
    assert call(n=131073) == HCU_ERR_ARG        # past the width the select's bitmaps cover
    assert call(wsb=1024) == HCU_ERR_ARG        # workspace too small
    assert call(workspace=None) == HCU_ERR_ARG
    assert call(pt_stride=-1) == HCU_ERR_ARG
    assert call(rows=0) == HCU_OK


def test_list_topk_workspace_and_argument_checks(lib):
    """The many-row list top-k: its workspace query (about 64 KiB a row, 256-byte multiples) and
    the checks it makes before launching anything."""
    ws = lib.hcu_sparse_mask_topk_transform_lists_workspace_bytes
    ws.restype = ctypes.c_int64
    ws.argtypes = [ctypes.c_int64, ctypes.c_int64]
    assert ws(-1, 10) == -1
    assert ws(8192, 73728) >= 8192 * 8192 * 8
    assert ws(8192, 73728) % 256 == 0
    f = lib.hcu_sparse_mask_topk_transform_lists
    f.restype = ctypes.c_int
    p, i64 = ctypes.c_void_p(256), ctypes.c_int64

    def call(rows=400, width=65536, topk=2048, wsb=None, workspace=p):
        b = ws(rows, width) if wsb is None else wsb
        return f(p, i64(rows), i64(width), i64(width), p, i64((width + 15) // 16), p, p, i64(width), i64(topk),
                 workspace, i64(b), p, None)

    assert call(topk=100) == HCU_ERR_ARG
    assert call(width=131072 + 16) == HCU_ERR_ARG  # past the width the select's bitmaps cover
    assert call(wsb=4096) == HCU_ERR_ARG           # workspace too small
    assert call(workspace=None) == HCU_ERR_ARG
    assert call(workspace=ctypes.c_void_p(272)) == HCU_ERR_ARG  # not 256-byte aligned
    assert call(rows=0) == HCU_OK
