// MLA decode front end in one launch: the q rope, the RMS norm of the 512-wide latent and its
// fp8 store into the 656-byte KV slot, and the k rope (hcu_ops.rope_qout_kv_store of the
// reference, hcu_ops/csrc/mla_kv.cu:1-13,85-170; the producer of the 656-byte slots that
// dequant_mla_kernel reads).
//
// grid = (T, ceil(nq / 8) + 1), 256 threads.  CTAs y < ceil(nq / 8): thread = one rotated pair of
// one q head (8 heads x 32 pairs).  The last CTA of token t:
//   * threads 0..63, 8 latent elements each: sum of squares (8 sequential fused multiply-adds,
//     then the reference's 64-lane tree: lane j < 32 adds lane j + 32, then offsets 16..1),
//     rstd = rsqrt(ss / 512 + eps) in the selected form, y = bf16((x * rstd) * w) written back in
//     place; then per 128-element group amax, scale = max(amax, store_eps) / 448 and the fp8
//     e4m3 bytes of y * (1 / scale) (round to nearest even, saturated) into the slot, the four
//     fp32 scales at +512;
//   * threads 64..95: the k rope pair, in place in k_pe and as bf16 at +528 of the slot.
// The rope follows the reference's bf16 arithmetic: every product and the difference / sum
// are rounded to bf16 (c10::BFloat16 operators), NaN -> 0x7FC0.  Rows t >= n_loc are normed
// and rotated but not stored.  A token whose position is outside the cos/sin cache is skipped
// entirely, and a slot outside the buffer is not written; both are flagged HCU_STATUS_BAD_INPUT.
#include <cuda_fp8.h>

#include "common.cuh"

HCU_DEFINE_STATUS(status_mla)

namespace hcu {
namespace {

constexpr int kNope = 512;
constexpr int kRot = 64;
constexpr int kSlotScale = kNope;               // 4 fp32 group scales
constexpr int kSlotRope = kNope + 4 * 4;        // 64 bf16
constexpr int kSlotBytes = kSlotRope + 2 * kRot;  // 656
constexpr int kMlaThreads = 256;
constexpr int kHeadsPerCta = kMlaThreads / (kRot / 2);

__device__ __forceinline__ float bf(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }

// float -> bf16, round to nearest even; NaN -> 0x7FC0 (c10::BFloat16's conversion)
__device__ __forceinline__ uint16_t to_bf(float f) {
  if (f != f) return 0x7FC0;
  const uint32_t u = __float_as_uint(f);
  return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// Rotated pair r of a 64-element row: (xi, yi) and their new bf16 values.
template <bool kNeox>
__device__ __forceinline__ void rope_pair(const uint16_t* src, const uint16_t* cs, int r, int& xi, int& yi,
                                          uint16_t& ox, uint16_t& oy) {
  xi = kNeox ? r : 2 * r;
  yi = kNeox ? kRot / 2 + r : 2 * r + 1;
  const float c = bf(cs[r]);
  const float s = bf(cs[kRot / 2 + r]);
  const float x = bf(src[xi]);
  const float y = bf(src[yi]);
  ox = to_bf(bf(to_bf(__fmul_rn(x, c))) - bf(to_bf(__fmul_rn(y, s))));
  oy = to_bf(bf(to_bf(__fmul_rn(y, c))) + bf(to_bf(__fmul_rn(x, s))));
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

template <typename PosT, bool kNeox, int kRsqrt>
__global__ __launch_bounds__(kMlaThreads) void rope_qout_kv_store_kernel(const MlaArgs p) {
  __shared__ float part[64];
  __shared__ float s_rstd;
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t pos = static_cast<int64_t>(reinterpret_cast<const PosT*>(p.positions)[t]);
  if (pos < 0 || pos >= p.n_pos) {  // uniform over the CTA
    if (tid == 0) atomicOr(&g_hcu_status, HCU_STATUS_BAD_INPUT);
    return;
  }
  const uint16_t* cs = p.cache + pos * kRot;
  int xi, yi;
  uint16_t ox, oy;

  if (blockIdx.y + 1 < gridDim.y) {  // q heads
    const int h = blockIdx.y * kHeadsPerCta + tid / (kRot / 2);
    if (h < p.nq) {
      rope_pair<kNeox>(p.q + t * p.q_tok + h * p.q_head, cs, tid % (kRot / 2), xi, yi, ox, oy);
      uint16_t* dst = p.qo + t * p.qo_tok + h * p.qo_head;
      dst[xi] = ox;
      dst[yi] = oy;
    }
    return;
  }

  bool store = t < p.n_loc;
  uint8_t* slot = nullptr;
  if (store) {
    const int64_t l = p.loc[t];
    if (l < 0 || l >= p.n_slots) {
      store = false;
      if (tid == 0) atomicOr(&g_hcu_status, HCU_STATUS_BAD_INPUT);
    } else {
      slot = p.kv + l * p.slot_stride;
    }
  }
  if (tid < 64) {
    const int lane = tid;
    uint16_t* row = p.kv_c + t * p.kv_tok + lane * 8;
    const uint4 rx = *reinterpret_cast<const uint4*>(row);
    const uint4 rw = __ldg(reinterpret_cast<const uint4*>(p.gamma + lane * 8));
    const uint16_t* hx = reinterpret_cast<const uint16_t*>(&rx);
    const uint16_t* hw = reinterpret_cast<const uint16_t*>(&rw);
    float x[8];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] = bf(hx[i]);
      sum = __fmaf_rn(x[i], x[i], sum);
    }
    part[lane] = sum;
    named_bar(1, 64);
    if (lane < 32) {  // the 64-lane tree: j += j + 32, then offsets 16, 8, 4, 2, 1
      float v = part[lane] + part[lane + 32];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
      if (lane == 0) {
        const float m = __fadd_rn(__fdiv_rn(v, static_cast<float>(kNope)), p.norm_eps);
        s_rstd = kRsqrt == 2 ? __fdiv_rn(1.f, __fsqrt_rn(m)) : rsqrtf(m);
      }
    }
    named_bar(1, 64);
    const float rstd = s_rstd;
    uint4 ry;
    uint16_t* hy = reinterpret_cast<uint16_t*>(&ry);
    float y[8];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      hy[i] = to_bf(__fmul_rn(__fmul_rn(x[i], rstd), bf(hw[i])));
      y[i] = bf(hy[i]);
      amax = fmaxf(amax, fabsf(y[i]));
    }
    *reinterpret_cast<uint4*>(row) = ry;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));  // 16-lane groups
    if (store) {
      amax = fmaxf(amax, p.store_eps);
      const float scale = __fdiv_rn(amax, 448.f);
      const float inv = scale == 0.f ? 0.f : __fdiv_rn(1.f, scale);
      if ((lane & 15) == 0) reinterpret_cast<float*>(slot + kSlotScale)[lane >> 4] = scale;
      uint32_t wv[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
            make_float2(__fmul_rn(y[4 * i], inv), __fmul_rn(y[4 * i + 1], inv)), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
            make_float2(__fmul_rn(y[4 * i + 2], inv), __fmul_rn(y[4 * i + 3], inv)), __NV_SATFINITE, __NV_E4M3);
        wv[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
      }
      *reinterpret_cast<uint2*>(slot + lane * 8) = make_uint2(wv[0], wv[1]);
    }
  } else if (tid < 64 + kRot / 2) {
    uint16_t* kr = p.k_pe + t * p.k_tok;
    rope_pair<kNeox>(kr, cs, tid - 64, xi, yi, ox, oy);
    kr[xi] = ox;
    kr[yi] = oy;
    if (store) {
      uint16_t* cr = reinterpret_cast<uint16_t*>(slot + kSlotRope);
      cr[xi] = ox;
      cr[yi] = oy;
    }
  }
}

template <typename PosT, bool kNeox>
void launch_mla(const MlaArgs& a, int64_t T, int rsqrt_mode, cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>(T), static_cast<unsigned>((a.nq + kHeadsPerCta - 1) / kHeadsPerCta + 1));
  if (rsqrt_mode == 2)
    rope_qout_kv_store_kernel<PosT, kNeox, 2><<<grid, kMlaThreads, 0, st>>>(a);
  else
    rope_qout_kv_store_kernel<PosT, kNeox, 0><<<grid, kMlaThreads, 0, st>>>(a);
}

bool al16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

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
  if (n_tokens < 0 || n_tokens > INT32_MAX || nq < 0 || nq > 65534 * kHeadsPerCta || n_loc < 0 || n_loc > n_tokens)
    return HCU_ERR_ARG;
  if (rsqrt_mode < 0 || rsqrt_mode > 2 || n_pos < 0 || n_slots < 0) return HCU_ERR_ARG;
  if (n_tokens == 0) return HCU_OK;
  if (!positions || (nq > 0 && (!q_pe || !q_out)) || !kv_c || !kv_weight || !k_pe || !cos_sin_cache)
    return HCU_ERR_ARG;
  if (n_loc > 0 && (!kv_buffer || !loc)) return HCU_ERR_ARG;
  // 16-byte latent rows and weight (one 16-B load per 8 elements), 16-byte slots (8-B fp8 stores,
  // fp32 scales at +512)
  if (!al16(kv_c) || kv_tok % 8 != 0 || kv_tok < kNope || !al16(kv_weight)) return HCU_ERR_ARG;
  if (n_loc > 0 && (!al16(kv_buffer) || slot_stride % 16 != 0 || slot_stride < kSlotBytes)) return HCU_ERR_ARG;
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
    is_neox ? launch_mla<int64_t, true>(a, n_tokens, rsqrt_mode, st) : launch_mla<int64_t, false>(a, n_tokens, rsqrt_mode, st);
  else
    is_neox ? launch_mla<int32_t, true>(a, n_tokens, rsqrt_mode, st) : launch_mla<int32_t, false>(a, n_tokens, rsqrt_mode, st);
  return launch_status();
}
