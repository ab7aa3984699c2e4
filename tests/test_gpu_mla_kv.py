"""GPU parity of the MLA decode front end (rope_qout_kv_store): q rope, RMS norm of the latent in
place, k rope, fp8 656-byte slot store, against its CPU restatement (``oracle/mla.py``).  Operands
are laid out as in the reference's own test (``hcu_ops/tests/test_kv_fused.py:18-46``): a packed
[T, 2048 + 576] latent (kv_c and k_pe are views into it), q [T, 64, 256] with the rope tail at 192,
q_out either q_pe itself or a view into q_cat [T, 64, 576]; outlier channels, a zero row, one huge
element, int32 and int64 positions, fewer slots than tokens.  With rsqrt_mode 2 (1 / sqrtf) every
byte is compared exactly; modes 0/1 (rsqrtf) allow one bf16 ulp in the normed latent and one fp8
code in the slot."""
import numpy as np
import pytest
import torch

from oracle import indexer as OI
from oracle import mla as O

pytestmark = pytest.mark.gpu

H, QL, KVL, ROT, SLOT = 64, 2048, 512, 64, 656
MAX_POS, SLOTS = 70000, 512


def _cache():
    ang = torch.arange(MAX_POS)[:, None] * (10000.0 ** (-torch.arange(ROT // 2) / (ROT // 2)))
    return torch.cat([ang.cos(), ang.sin()], dim=-1).bfloat16().contiguous()


def _make(t, seed):
    g = torch.Generator().manual_seed(seed)
    packed = torch.randn(t, QL + KVL + ROT, generator=g).bfloat16()
    packed[:, QL:QL + KVL:37] *= 16  # outlier channels
    if t > 2:
        packed[1, QL:QL + KVL] = 0  # zero row: rstd = rsqrt(eps), amax 0 -> store_eps
    if t > 3:
        packed[2, QL + 5] = 3e4  # one huge element
    q = torch.randn(t, H, 256, generator=g).bfloat16()
    pos = torch.randint(0, MAX_POS, (t,), generator=g)
    w = (torch.rand(KVL, generator=g) * 2).bfloat16()
    return packed, q, pos, w


def _u16(x):
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


def _run(hcu, dev, t, eps, neox, inplace, pos32, short_loc, mode, seed):
    import hcu_ops

    packed, q, pos, w = _make(t, seed)
    cache = _cache()
    n_loc = t - 1 if short_loc and t > 1 else t
    g = torch.Generator().manual_seed(seed + 1)
    loc = torch.randperm(SLOTS, generator=g)[:n_loc].contiguous()
    buf = torch.randint(0, 256, (SLOTS, 1, SLOT), generator=g, dtype=torch.uint8)
    ref = O.rope_qout_kv_store(pos.numpy(), _u16(q[..., 192:]), _u16(packed[:, QL:QL + KVL]), _u16(w), eps,
                               _u16(packed[:, QL + KVL:]), _u16(cache), neox, buf.numpy(), loc.numpy())
    P, Q, W, C, B, L = (x.to(dev) for x in (packed, q, w, cache, buf, loc))
    Pp = (pos.int() if pos32 else pos).to(dev)
    kv_c, k_pe, q_pe = P[:, QL:QL + KVL], P[:, QL + KVL:].unsqueeze(1), Q[..., 192:]
    q_cat = q_pe if inplace else torch.zeros(t, H, KVL + ROT, dtype=torch.bfloat16, device=dev)
    q_out = q_pe if inplace else q_cat[..., KVL:]
    assert hcu_ops.kv_fused_supported(Pp, q_pe, q_out, kv_c, W, k_pe, C, B, L)
    hcu._C.rope_qout_kv_store(Pp, q_pe, q_out, kv_c, W, eps, k_pe, C, neox, B, L, 1e-6, mode)
    torch.cuda.synchronize()
    return ref, (packed, q), (P.cpu(), Q.cpu(), q_cat.cpu(), B.cpu())


CASES = [(1, 1e-6, False, False, False, False), (3, 1e-5, True, True, True, True),
         (5, 1e-6, True, False, True, True), (16, 1e-6, False, True, False, False),
         (33, 1e-5, False, False, True, True), (128, 1e-6, True, False, False, False)]


@pytest.mark.parametrize("mode", [2, 0])
@pytest.mark.parametrize("case", CASES, ids=[f"T{c[0]}-neox{int(c[2])}-inpl{int(c[3])}" for c in CASES])
def test_rope_qout_kv_store_matches_restatement(hcu, dev, mode, case):
    t, eps, neox, inplace, pos32, short_loc = case
    (q_out_r, kv_r, kp_r, buf_r), (packed0, q0), (P, Q, q_cat, B) = _run(hcu, dev, t, eps, neox, inplace, pos32,
                                                                         short_loc, mode, seed=t)
    # untouched: the q-lora part of the latent and q's nope part
    assert torch.equal(P[:, :QL], packed0[:, :QL])
    assert torch.equal(Q[..., :192], q0[..., :192])
    # the ropes do not depend on the norm: exact in every mode
    assert np.array_equal(_u16(P[:, QL + KVL:]), kp_r)
    got_q = _u16(Q[..., 192:]) if inplace else _u16(q_cat[..., KVL:])
    assert np.array_equal(got_q, q_out_r)
    if not inplace:
        assert (q_cat[..., :KVL] == 0).all()
    kv = _u16(P[:, QL:QL + KVL])
    b = B.numpy().reshape(SLOTS, SLOT)
    r = buf_r.reshape(SLOTS, SLOT)
    if mode == 2:
        assert np.array_equal(kv, kv_r)
        assert np.array_equal(b, r)
        return
    # rsqrtf: the normed latent within one bf16 ulp, the slot's fp8 codes within one, scales within 2^-7
    d = np.abs(kv.astype(np.int32) - kv_r.astype(np.int32))
    assert d.max() <= 1, int(d.max())
    assert np.array_equal(b[:, 528:], r[:, 528:])  # rope copy
    same = b[:, :512] == r[:, :512]  # unwritten slots keep their (random) bytes on both sides
    fp = np.abs(OI.e4m3_to_f32(b[:, :512]) - OI.e4m3_to_f32(r[:, :512]))
    step = np.abs(OI.e4m3_to_f32(r[:, :512])) / 8 + 2.0 ** -9
    assert (same | (fp <= step)).all()
    sg, sr = b[:, 512:528].copy().view(np.float32), r[:, 512:528].copy().view(np.float32)
    assert ((b[:, 512:528] == r[:, 512:528]).reshape(SLOTS, 4, 4).all(axis=2) | np.isclose(sg, sr, rtol=2.0 ** -7, atol=0)).all()


def test_slot_dequantizes_to_the_normed_latent(hcu, dev):
    """The written slots read back through dequant_mla_656 (the consumer of this layout): the fp8
    part within fp8 precision of the normed latent, the rope part bit-exact."""
    t = 40
    (q_out_r, kv_r, kp_r, buf_r), _, (P, Q, q_cat, B) = _run(hcu, dev, t, 1e-6, False, False, False, False, 2, 5)
    g = torch.Generator().manual_seed(6)
    loc = torch.randperm(SLOTS, generator=g)[:t].contiguous()
    out = hcu.dequantize_k_cache_paged(B.to(dev), loc.to(torch.int32).to(dev)).cpu()
    y = O.bf(_u16(P[:, QL:QL + KVL]))
    deq = out.view(t, 576)[:, :512].float().numpy()
    # per 128-element group: relative fp8 precision, plus half the smallest subnormal step of its scale
    scale = np.maximum(np.abs(y).reshape(t, 4, 128).max(axis=2), 1e-6) / 448
    atol = np.repeat(scale, 128, axis=1) * 2.0 ** -9
    assert (np.abs(deq - y) <= 2.0 ** -4 * np.abs(y) + atol).all()
    assert np.array_equal(_u16(out.view(t, 576)[:, 512:]), _u16(P[:, QL + KVL:]))


def test_bad_position_and_slot_are_skipped_and_flagged(hcu, dev, request):
    request.node.allowed_status = 2  # HCU_STATUS_BAD_INPUT
    t = 4
    packed, q, pos, w = _make(t, 9)
    pos[1] = MAX_POS + 5  # outside the cos/sin cache: token 1 untouched
    cache = _cache()
    loc = torch.tensor([3, 7, SLOTS + 1, 9])  # token 2's slot outside the buffer: not written
    buf = torch.zeros(SLOTS, 1, SLOT, dtype=torch.uint8)
    P, Q, W, C, B, L, Pp = (x.to(dev) for x in (packed, q, w, cache, buf, loc, pos))
    kv_c, k_pe, q_pe = P[:, QL:QL + KVL], P[:, QL + KVL:].unsqueeze(1), Q[..., 192:]
    hcu._C.rope_qout_kv_store(Pp, q_pe, q_pe, kv_c, W, 1e-6, k_pe, C, False, B, L, 1e-6, 2)
    assert hcu.read_device_status(clear=False) & 2
    P, Q, B = P.cpu(), Q.cpu(), B.cpu()
    assert torch.equal(P[1], packed[1]) and torch.equal(Q[1], q[1])
    assert (B[7] == 0).all() and (B[SLOTS - 1] == 0).all()
    assert not torch.equal(P[2, QL:QL + KVL], packed[2, QL:QL + KVL])  # token 2 normed all the same
    assert (B[3] != 0).any() and (B[9] != 0).any()
