// MLA decode front end in one launch (hcu_ops.rope_qout_kv_store of the reference,
// hcu_ops/csrc/mla_kv.cu:1-13,85; the producer of the 656-byte slots that dequant_mla_kernel
// reads): the rope of every q head, the RMS norm of the 512-wide latent written back in place and
// its fp8 store into the slot, and the rope of k_pe (in place and into the slot).
//
// One 256-thread CTA per token (8 warps):
//   * warp 0 owns the latent: lane l holds the 16 consecutive elements [16 l, 16 l + 16) (two
//     16-byte loads), so the whole norm, quantisation and store happen in registers and shuffles
//     of one warp, with no shared memory and no CTA barrier;
//   * warps 1..7 own "rope units": a unit is 4 consecutive rotation pairs of one 64-element row,
//     eight units per row, and the rows are the nq q heads followed by k_pe.  A unit reads its
//     pairs' elements and cos / sin with 8- or 16-byte accesses (one 16-byte access per unit for
//     the interleaved layout, two 8-byte ones for neox) and writes the rotated values back.
//
// Arithmetic contract (bit-exact against the reference's rounding steps):
//   * sum of squares: the reference reduces 64 partial sums p[j] of 8 consecutive elements (each a
//     chain of fused multiply-adds) as v[j] = p[j] + p[j + 32] for j < 32, then v[j] += v[j + o]
//     for o = 16, 8, 4, 2, 1.  Lane l holds p[2l] and p[2l + 1]; the same additions are done
//     pairwise across lanes (see norm_warp);
//   * rstd = 1 / sqrt(ss / 512 + eps) (IEEE, rsqrt mode 2) or rsqrtf (modes 0 and 1);
//     y = bf16((x * rstd) * w);
//   * per 128-element group: scale = max(amax, store_eps) / 448, fp8 e4m3 of y * (1 / scale)
//     (round to nearest even, saturated to +-448);
//   * rope in bf16 arithmetic: every product and the difference / sum rounded to bf16 (c10
//     BFloat16 operators; NaN becomes 0x7FC0).
// Rows t >= n_loc are normed and rotated but not stored.  A token whose position is outside the
// cos/sin cache is skipped entirely and a slot outside the buffer is not written (the reference
// reads / writes out of range there); both set HCU_STATUS_BAD_INPUT.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "common.cuh"

HCU_DEFINE_STATUS(status_mla)

namespace hcu {
namespace {

constexpr int kLatent = 512;
constexpr int kRope = 64;
constexpr int kPairs = kRope / 2;
constexpr int kScaleOff = kLatent;                // 4 fp32 group scales
constexpr int kRopeOff = kLatent + 16;            // 64 bf16, 16-byte aligned
constexpr int kSlotBytes = kRopeOff + 2 * kRope;  // 656
constexpr int kThreads = 256;
constexpr int kUnitsPerRow = kPairs / 4;          // 8 units of 4 pairs
constexpr int kUnitThreads = kThreads - 32;       // warps 1..7
constexpr int kBatch = 3;                         // units per thread in flight (65 rows x 8 units <= 3 x 224)

__device__ __forceinline__ float bf2f(uint32_t h16) { return __uint_as_float(h16 << 16); }

// Round to nearest even through the hardware conversion; NaN gets c10's canonical 0x7FC0.
__device__ __forceinline__ uint32_t f2bf(float f) {
  return f != f ? 0x7FC0u : static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(f)));
}

// (x, y) -> (x c - y s, y c + x s) with each product and the sum / difference rounded to bf16.
__device__ __forceinline__ void rotate(uint32_t xb, uint32_t yb, uint32_t cb, uint32_t sb, uint32_t& ox,
                                       uint32_t& oy) {
  const float x = bf2f(xb), y = bf2f(yb), c = bf2f(cb), s = bf2f(sb);
  const float xc = bf2f(f2bf(__fmul_rn(x, c))), ys = bf2f(f2bf(__fmul_rn(y, s)));
  const float yc = bf2f(f2bf(__fmul_rn(y, c))), xs = bf2f(f2bf(__fmul_rn(x, s)));
  ox = f2bf(xc - ys);
  oy = f2bf(yc + xs);
}

struct MlaArgs {
  const void* positions;
  const uint16_t* q;
  uint16_t* qo;
  int64_t q_tok, q_head, qo_tok, qo_head;
  uint16_t* kv_c;
  int64_t kv_tok;
  const uint16_t* gamma;
  float norm_eps;
  uint16_t* k_pe;
  int64_t k_tok;
  const uint16_t* cache;
  int64_t n_pos;
  uint8_t* kv;
  int64_t n_slots, slot_stride;
  const int64_t* loc;
  int nq, n_loc;
  float store_eps;
};

__device__ __forceinline__ void unpack8(const uint4& v, uint32_t (&h)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    h[2 * i] = w[i] & 0xFFFFu;
    h[2 * i + 1] = w[i] >> 16;
  }
}

__device__ __forceinline__ uint4 pack8(const uint32_t (&h)[8]) {
  return make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
}

// Warp 0: RMS norm of the latent row in place and (slot != null) its fp8 groups and scales.
template <int kRsqrt>
__device__ __forceinline__ void norm_warp(const MlaArgs& p, int64_t t, uint8_t* slot) {
  const int lane = threadIdx.x & 31;
  uint16_t* row = p.kv_c + t * p.kv_tok + 16 * lane;
  uint32_t x[16], g[16];
  {
    uint32_t a[8], b[8];
    unpack8(*reinterpret_cast<const uint4*>(row), a);
    unpack8(*reinterpret_cast<const uint4*>(row + 8), b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] = a[i];
      x[8 + i] = b[i];
    }
    unpack8(__ldg(reinterpret_cast<const uint4*>(p.gamma + 16 * lane)), a);
    unpack8(__ldg(reinterpret_cast<const uint4*>(p.gamma + 16 * lane + 8)), b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      g[i] = a[i];
      g[8 + i] = b[i];
    }
  }
  // partial sums p[2l] (elements 16l..16l+7) and p[2l+1] (16l+8..16l+15)
  float e = 0.f, o = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float xe = bf2f(x[i]), xo = bf2f(x[8 + i]);
    e = __fmaf_rn(xe, xe, e);
    o = __fmaf_rn(xo, xo, o);
  }
  // v[j] = p[j] + p[j + 32], held as v[2l], v[2l + 1] on lanes l < 16 (p[j + 32] is on lane l + 16);
  // then v[j] += v[j + 16], += v[j + 8], ... : lane l adds lane l + 8, l + 4, l + 2, l + 1's pair, and
  // the last step (v[0] += v[1]) adds the two halves of lane 0's pair.
  e += __shfl_down_sync(0xffffffffu, e, 16);
  o += __shfl_down_sync(0xffffffffu, o, 16);
#pragma unroll
  for (int d = 8; d >= 1; d >>= 1) {
    e += __shfl_down_sync(0xffffffffu, e, d);
    o += __shfl_down_sync(0xffffffffu, o, d);
  }
  const float ss = __shfl_sync(0xffffffffu, e + o, 0);
  const float m = __fadd_rn(__fdiv_rn(ss, static_cast<float>(kLatent)), p.norm_eps);
  const float rstd = kRsqrt == 2 ? __fdiv_rn(1.f, __fsqrt_rn(m)) : rsqrtf(m);
  uint32_t y[16];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    y[i] = f2bf(__fmul_rn(__fmul_rn(bf2f(x[i]), rstd), bf2f(g[i])));
    amax = fmaxf(amax, fabsf(bf2f(y[i])));  // fmaxf drops NaN, as the reference's amax loop
  }
  {
    uint32_t a[8], b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      a[i] = y[i];
      b[i] = y[8 + i];
    }
    *reinterpret_cast<uint4*>(row) = pack8(a);
    *reinterpret_cast<uint4*>(row + 8) = pack8(b);
  }
  if (slot == nullptr) return;
  // group q = lanes [8q, 8q + 8): four warp max-reductions of the (non-negative, non-NaN) amax bits
  const int grp = lane >> 3;
  const uint32_t ab = __float_as_uint(amax);
  float sc[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float gmax = __uint_as_float(__reduce_max_sync(0xffffffffu, grp == q ? ab : 0u));
    sc[q] = __fdiv_rn(fmaxf(gmax, p.store_eps), 448.f);
  }
  if (lane == 0) *reinterpret_cast<float4*>(slot + kScaleOff) = make_float4(sc[0], sc[1], sc[2], sc[3]);
  const float s = grp == 0 ? sc[0] : (grp == 1 ? sc[1] : (grp == 2 ? sc[2] : sc[3]));
  const float inv = s == 0.f ? 0.f : __fdiv_rn(1.f, s);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
        make_float2(__fmul_rn(bf2f(y[4 * i]), inv), __fmul_rn(bf2f(y[4 * i + 1]), inv)), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
        make_float2(__fmul_rn(bf2f(y[4 * i + 2]), inv), __fmul_rn(bf2f(y[4 * i + 3]), inv)), __NV_SATFINITE,
        __NV_E4M3);
    w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
  *reinterpret_cast<uint4*>(slot + 16 * lane) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Element indices of pair r: interleaved (2r, 2r + 1), neox (r, r + 32).
template <bool kNeox>
__device__ __forceinline__ int px(int r) { return kNeox ? r : 2 * r; }
template <bool kNeox>
__device__ __forceinline__ int py(int r) { return kNeox ? kPairs + r : 2 * r + 1; }

// The inputs of one rope unit (pairs 4u .. 4u + 3 of a 64-element row) as loaded: interleaved
// w[i] = x_i | y_i << 16; neox w[0..1] = x_0..x_3 and w[2..3] = y_0..y_3 (two bf16 per word);
// c, s: cos_0..3 and sin_0..3 two per word.
struct RopeIn {
  uint32_t w[4];
  uint32_t c[2], s[2];
};

__device__ __forceinline__ uint32_t pack2(uint32_t lo, uint32_t hi) { return (lo & 0xFFFFu) | (hi << 16); }

template <bool kNeox, bool kVec>
__device__ __forceinline__ RopeIn rope_load(const uint16_t* src, const uint16_t* cs, int u) {
  RopeIn in;
  if constexpr (kVec) {
    const uint2 cv = __ldg(reinterpret_cast<const uint2*>(cs + 4 * u));
    const uint2 sv = __ldg(reinterpret_cast<const uint2*>(cs + kPairs + 4 * u));
    in.c[0] = cv.x; in.c[1] = cv.y;
    in.s[0] = sv.x; in.s[1] = sv.y;
    if constexpr (kNeox) {
      const uint2 a = *reinterpret_cast<const uint2*>(src + 4 * u);
      const uint2 b = *reinterpret_cast<const uint2*>(src + kPairs + 4 * u);
      in.w[0] = a.x; in.w[1] = a.y; in.w[2] = b.x; in.w[3] = b.y;
    } else {
      const uint4 a = *reinterpret_cast<const uint4*>(src + 8 * u);
      in.w[0] = a.x; in.w[1] = a.y; in.w[2] = a.z; in.w[3] = a.w;
    }
  } else {
    const int r = 4 * u;
    in.c[0] = pack2(cs[r], cs[r + 1]);
    in.c[1] = pack2(cs[r + 2], cs[r + 3]);
    in.s[0] = pack2(cs[kPairs + r], cs[kPairs + r + 1]);
    in.s[1] = pack2(cs[kPairs + r + 2], cs[kPairs + r + 3]);
    if constexpr (kNeox) {
      in.w[0] = pack2(src[r], src[r + 1]);
      in.w[1] = pack2(src[r + 2], src[r + 3]);
      in.w[2] = pack2(src[kPairs + r], src[kPairs + r + 1]);
      in.w[3] = pack2(src[kPairs + r + 2], src[kPairs + r + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) in.w[i] = pack2(src[2 * (r + i)], src[2 * (r + i) + 1]);
    }
  }
  return in;
}

// Rotates a loaded unit and stores it to dst (may alias the source row) and, when given, dst2.
template <bool kNeox, bool kVec>
__device__ __forceinline__ void rope_store(const RopeIn& in, uint16_t* dst, uint16_t* dst2, int u) {
  uint32_t x[4], y[4];
  if constexpr (kNeox) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[i] = (in.w[i >> 1] >> (16 * (i & 1))) & 0xFFFFu;
      y[i] = (in.w[2 + (i >> 1)] >> (16 * (i & 1))) & 0xFFFFu;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[i] = in.w[i] & 0xFFFFu;
      y[i] = in.w[i] >> 16;
    }
  }
  uint32_t ox[4], oy[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    rotate(x[i], y[i], (in.c[i >> 1] >> (16 * (i & 1))) & 0xFFFFu, (in.s[i >> 1] >> (16 * (i & 1))) & 0xFFFFu,
           ox[i], oy[i]);
  if constexpr (kVec) {
    if constexpr (kNeox) {
      const uint2 a = make_uint2(ox[0] | (ox[1] << 16), ox[2] | (ox[3] << 16));
      const uint2 b = make_uint2(oy[0] | (oy[1] << 16), oy[2] | (oy[3] << 16));
      *reinterpret_cast<uint2*>(dst + 4 * u) = a;
      *reinterpret_cast<uint2*>(dst + kPairs + 4 * u) = b;
      if (dst2) {
        *reinterpret_cast<uint2*>(dst2 + 4 * u) = a;
        *reinterpret_cast<uint2*>(dst2 + kPairs + 4 * u) = b;
      }
    } else {
      const uint4 a = make_uint4(ox[0] | (oy[0] << 16), ox[1] | (oy[1] << 16), ox[2] | (oy[2] << 16),
                                 ox[3] | (oy[3] << 16));
      *reinterpret_cast<uint4*>(dst + 8 * u) = a;
      if (dst2) *reinterpret_cast<uint4*>(dst2 + 8 * u) = a;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 4 * u + i;
      dst[px<kNeox>(r)] = static_cast<uint16_t>(ox[i]);
      dst[py<kNeox>(r)] = static_cast<uint16_t>(oy[i]);
      if (dst2) {
        dst2[px<kNeox>(r)] = static_cast<uint16_t>(ox[i]);
        dst2[py<kNeox>(r)] = static_cast<uint16_t>(oy[i]);
      }
    }
  }
}

template <typename PosT, bool kNeox, bool kVec, int kRsqrt>
__global__ __launch_bounds__(kThreads) void rope_qout_kv_store_kernel(const MlaArgs p) {
  const int64_t t = blockIdx.x;
  const int64_t pos = static_cast<int64_t>(reinterpret_cast<const PosT*>(p.positions)[t]);
  if (pos < 0 || pos >= p.n_pos) {  // the whole CTA skips the token
    if (threadIdx.x == 0) atomicOr(&g_hcu_status, HCU_STATUS_BAD_INPUT);
    return;
  }
  uint8_t* slot = nullptr;
  if (t < p.n_loc) {
    const int64_t l = p.loc[t];
    if (l >= 0 && l < p.n_slots)
      slot = p.kv + l * p.slot_stride;
    else if (threadIdx.x == 0)
      atomicOr(&g_hcu_status, HCU_STATUS_BAD_INPUT);
  }
  if (threadIdx.x < 32) {
    norm_warp<kRsqrt>(p, t, slot);
    return;
  }
  const uint16_t* cs = p.cache + pos * kRope;
  const int units = (p.nq + 1) * kUnitsPerRow;  // q heads, then k_pe
  // each thread loads up to kBatch units before rotating any, so their loads are in flight together
  // (a unit's stores may alias its own source elements only, never another unit's)
  for (int v0 = static_cast<int>(threadIdx.x) - 32; v0 < units; v0 += kBatch * kUnitThreads) {
    RopeIn in[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int v = v0 + b * kUnitThreads;
      if (v < units) {
        const int h = v / kUnitsPerRow;
        const int u = v - h * kUnitsPerRow;
        const uint16_t* src = h < p.nq ? p.q + t * p.q_tok + h * p.q_head : p.k_pe + t * p.k_tok;
        in[b] = rope_load<kNeox, kVec>(src, cs, u);
      }
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int v = v0 + b * kUnitThreads;
      if (v < units) {
        const int h = v / kUnitsPerRow;
        const int u = v - h * kUnitsPerRow;
        if (h < p.nq)
          rope_store<kNeox, kVec>(in[b], p.qo + t * p.qo_tok + h * p.qo_head, nullptr, u);
        else
          rope_store<kNeox, kVec>(in[b], p.k_pe + t * p.k_tok,
                                  slot ? reinterpret_cast<uint16_t*>(slot + kRopeOff) : nullptr, u);
      }
    }
  }
}

template <typename PosT, bool kNeox, bool kVec>
void launch_mla(const MlaArgs& a, int64_t T, int rsqrt_mode, cudaStream_t st) {
  if (rsqrt_mode == 2)
    rope_qout_kv_store_kernel<PosT, kNeox, kVec, 2><<<static_cast<unsigned>(T), kThreads, 0, st>>>(a);
  else
    rope_qout_kv_store_kernel<PosT, kNeox, kVec, 0><<<static_cast<unsigned>(T), kThreads, 0, st>>>(a);
}

template <typename PosT, bool kNeox>
void launch_layout(const MlaArgs& a, int64_t T, int rsqrt_mode, bool vec, cudaStream_t st) {
  vec ? launch_mla<PosT, kNeox, true>(a, T, rsqrt_mode, st) : launch_mla<PosT, kNeox, false>(a, T, rsqrt_mode, st);
}

bool aligned(const void* p, uintptr_t n) { return reinterpret_cast<uintptr_t>(p) % n == 0; }

}  // namespace
}  // namespace hcu

extern "C" int hcu_rope_qout_kv_store(const void* positions, int32_t positions_int64, int64_t n_tokens,
                                      const uint16_t* q_pe, int64_t nq, int64_t q_tok, int64_t q_head,
                                      uint16_t* q_out, int64_t qo_tok, int64_t qo_head, uint16_t* kv_c,
                                      int64_t kv_tok, const uint16_t* kv_weight, float norm_eps, uint16_t* k_pe,
                                      int64_t k_tok, const uint16_t* cos_sin_cache, int64_t n_pos, int32_t is_neox,
                                      uint8_t* kv_buffer, int64_t n_slots, int64_t slot_stride, const int64_t* loc,
                                      int64_t n_loc, float store_eps, int32_t rsqrt_mode, hcu_stream_t stream) {
  using namespace hcu;
  if (n_tokens < 0 || n_tokens > INT32_MAX || nq < 0 || nq > (1 << 20) || n_loc < 0 || n_loc > n_tokens)
    return HCU_ERR_ARG;
  if (rsqrt_mode < 0 || rsqrt_mode > 2 || n_pos < 0 || n_slots < 0) return HCU_ERR_ARG;
  if (n_tokens == 0) return HCU_OK;
  if (!positions || (nq > 0 && (!q_pe || !q_out)) || !kv_c || !kv_weight || !k_pe || !cos_sin_cache)
    return HCU_ERR_ARG;
  if (n_loc > 0 && (!kv_buffer || !loc)) return HCU_ERR_ARG;
  // latent rows and weight read as 16-byte vectors; slots written with 16-byte stores
  if (!aligned(kv_c, 16) || kv_tok % 8 != 0 || kv_tok < kLatent || !aligned(kv_weight, 16)) return HCU_ERR_ARG;
  if (n_loc > 0 && (!aligned(kv_buffer, 16) || slot_stride % 16 != 0 || slot_stride < kSlotBytes)) return HCU_ERR_ARG;
  // rope units use 16-byte (interleaved) or 8-byte (neox) accesses when every row start allows them
  const uintptr_t va = is_neox ? 8 : 16;
  const int64_t ve = static_cast<int64_t>(va / 2);
  const bool vec = aligned(k_pe, va) && k_tok % ve == 0 && aligned(cos_sin_cache, 8) &&
                   (nq == 0 || (aligned(q_pe, va) && aligned(q_out, va) && q_tok % ve == 0 && q_head % ve == 0 &&
                                qo_tok % ve == 0 && qo_head % ve == 0));
  MlaArgs a;
  a.positions = positions;
  a.q = q_pe;
  a.qo = q_out;
  a.q_tok = q_tok;
  a.q_head = q_head;
  a.qo_tok = qo_tok;
  a.qo_head = qo_head;
  a.kv_c = kv_c;
  a.kv_tok = kv_tok;
  a.gamma = kv_weight;
  a.norm_eps = norm_eps;
  a.k_pe = k_pe;
  a.k_tok = k_tok;
  a.cache = cos_sin_cache;
  a.n_pos = n_pos;
  a.kv = kv_buffer;
  a.n_slots = n_slots;
  a.slot_stride = slot_stride;
  a.loc = loc;
  a.nq = static_cast<int>(nq);
  a.n_loc = static_cast<int>(n_loc);
  a.store_eps = store_eps;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (positions_int64)
    is_neox ? launch_layout<int64_t, true>(a, n_tokens, rsqrt_mode, vec, st)
            : launch_layout<int64_t, false>(a, n_tokens, rsqrt_mode, vec, st);
  else
    is_neox ? launch_layout<int32_t, true>(a, n_tokens, rsqrt_mode, vec, st)
            : launch_layout<int32_t, false>(a, n_tokens, rsqrt_mode, vec, st);
  return launch_status();
}
