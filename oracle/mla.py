"""CPU restatement of the MLA decode front end (test infrastructure only).

Restates ``hcu_ops/csrc/mla_kv.cu`` of the reference (``rope_qout_kv_store``): the q rope, the
RMS norm of the 512-wide latent, its fp8 store into the 656-byte slot and the k rope, in numpy
float32 with the reference's rounding steps.  Only ``tests/`` import it.  Parity: the reference's
kernel is HIP for gfx938 and its own test compares against lightop (absent here), so the
restatement follows the source line by line rather than pinned outputs.
"""
from __future__ import annotations

import numpy as np
import torch

NOPE, ROT, SLOT_SCALE, SLOT_ROPE, SLOT_BYTES = 512, 64, 512, 528, 656


def bf(u: np.ndarray) -> np.ndarray:
    """bf16 bits -> float32."""
    return (np.asarray(u, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_bf(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even, NaN -> 0x7FC0 (c10::BFloat16, ``mla_kv.cu:39-43``)."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), r)


def _rope(rows: np.ndarray, cs: np.ndarray, neox: bool) -> np.ndarray:
    """rope of bf16 rows [..., 64] with per-row cos/sin [..., 64] (32 cos then 32 sin), every product
    and the difference / sum rounded to bf16 (``mla_kv.cu:62-82``: c10::BFloat16 operators)."""
    r = np.arange(ROT // 2)
    xi, yi = (r, ROT // 2 + r) if neox else (2 * r, 2 * r + 1)
    c = bf(cs[..., :ROT // 2])
    s = bf(cs[..., ROT // 2:])
    x = bf(rows[..., xi])
    y = bf(rows[..., yi])
    out = np.array(rows, dtype=np.uint16, copy=True)
    out[..., xi] = to_bf(bf(to_bf(x * c)) - bf(to_bf(y * s)))
    out[..., yi] = to_bf(bf(to_bf(y * c)) + bf(to_bf(x * s)))
    return out


def _rstd(x: np.ndarray, eps: float) -> np.ndarray:
    """rsqrt(sum(x^2) / 512 + eps) per row, summed like ``mla_kv.cu:118-130``: 64 lanes of 8
    elements, each a sequential fused multiply-add, then lane j < 32 adds lane j + 32 and a tree
    over offsets 16..1 to lane 0; 1 / sqrt in IEEE float32 (rsqrt_mode 2)."""
    T = x.shape[0]
    lanes = x.reshape(T, 64, 8).astype(np.float64)
    s = np.zeros((T, 64), np.float32)
    for i in range(8):  # fma(x, x, s): the square is exact in float64, one rounding to float32
        s = (lanes[:, :, i] * lanes[:, :, i] + s.astype(np.float64)).astype(np.float32)
    v = (s[:, :32] + s[:, 32:]).astype(np.float32)
    for o in (16, 8, 4, 2, 1):
        v = np.concatenate([(v[:, :32 - o] + v[:, o:32]).astype(np.float32), v[:, 32 - o:]], axis=1)
    m = (v[:, 0] / np.float32(NOPE)).astype(np.float32) + np.float32(eps)
    return (np.float32(1.0) / np.sqrt(m.astype(np.float32))).astype(np.float32)


def rope_qout_kv_store(positions, q_pe, kv_c, kv_weight, norm_eps, k_pe, cos_sin_cache, is_neox, kv_buffer, loc,
                       store_eps=1e-6):
    """Returns (q_out, kv_c, k_pe, kv_buffer) after the op: bf16 bits (uint16) for the first three,
    ``[T, nq, 64]``, ``[T, 512]``, ``[T, 64]``; a written copy of the uint8 ``[slots, >= 656]``
    buffer.  Rows t >= len(loc) are normed and rotated but not stored (``mla_kv.cu:102-104``)."""
    pos = np.asarray(positions, dtype=np.int64)
    cache = np.asarray(cos_sin_cache, dtype=np.uint16)
    cs = cache[pos]                                             # [T, 64]
    q_out = _rope(np.asarray(q_pe, dtype=np.uint16), cs[:, None, :], is_neox)
    kp = _rope(np.asarray(k_pe, dtype=np.uint16), cs, is_neox)
    x = bf(np.asarray(kv_c, dtype=np.uint16))                  # [T, 512]
    w = bf(np.asarray(kv_weight, dtype=np.uint16))
    rstd = _rstd(x, norm_eps)
    yb = to_bf(((x * rstd[:, None]).astype(np.float32) * w[None, :]).astype(np.float32))
    y = bf(yb)
    buf = np.array(kv_buffer, dtype=np.uint8, copy=True)
    slots = buf.reshape(buf.shape[0], -1)                       # [slots, >= 656] (a view)
    loc = np.asarray(loc, dtype=np.int64)
    for t in range(loc.shape[0]):
        g = y[t].reshape(4, 128)
        amax = np.maximum(np.abs(g).max(axis=1), np.float32(store_eps)).astype(np.float32)
        scale = (amax / np.float32(448.0)).astype(np.float32)
        inv = np.where(scale == 0, np.float32(0), np.float32(1.0) / scale).astype(np.float32)
        v = np.clip((g * inv[:, None]).astype(np.float32), np.float32(-448.0), np.float32(448.0))
        q8 = torch.from_numpy(np.ascontiguousarray(v.reshape(-1))).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        slot = slots[int(loc[t])]
        slot[:NOPE] = q8
        slot[SLOT_SCALE:SLOT_SCALE + 16] = np.frombuffer(scale.tobytes(), np.uint8)
        slot[SLOT_ROPE:SLOT_ROPE + 2 * ROT] = np.frombuffer(kp[t].tobytes(), np.uint8)
    return q_out, yb, kp, buf
