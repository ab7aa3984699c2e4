// Stage 1: paged fp8 K-cache dequant (HBM streams).
//
// dequant_mla_kernel: the 656-byte MLA slot of sglang's DSA backend
//   (512 fp8 e4m3 | 4 fp32 group scales | 64 bf16 rope) -> 576 bf16, one warp
//   per token: lane l converts bytes [16l, 16l+16) with the scale of group l/8
//   and stores 32 contiguous output bytes; lanes 0-7 copy the rope.  Semantics
//   of prefill/patches/patch_fast_dequant.py:53-71 (fp32 multiply, one
//   round-to-nearest-even to bf16, rope copied bit for bit).
// dequant_index_k_kernel: the indexer-K page (64 x 128 fp8, then 64 fp32
//   scales) -> bf16 [n, 128]; 8 lanes per token, 4 tokens per warp access.
//
// quant_store_index_k_kernel: the writer of that page layout: per token
//   scale = max(amax, 1e-12) / 448 and fp8 e4m3 of x / scale (the correctly
//   rounded quotient, from one reciprocal per token and an FMA correction per
//   value; saturating round-to-nearest-even conversion), 8 lanes per token.
//
// All issue every load of kUnroll tokens before the first store so that each
// warp keeps several KB in flight (HBM latency x bandwidth per SM is ~40 KB).
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "common.cuh"

HCU_DEFINE_STATUS(status_dequant)

namespace hcu {
namespace {

constexpr int kMlaSlot = 656;
constexpr int kMlaOut = 576;
constexpr int kDqThreads = 256;
constexpr int kMlaUnroll = 4;
constexpr int kIdxUnroll = 4;

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Two fp8 e4m3 (low byte first) -> two bf16 of fp32(fp8) * s, packed.
__device__ __forceinline__ uint32_t cvt2(uint16_t two, float s) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two), __NV_E4M3);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  const float a = __fmul_rn(f.x, s);
  const float b = __fmul_rn(f.y, s);
  const __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&r);
}

// 16 fp8 bytes -> 32 output bytes.
__device__ __forceinline__ void cvt16(const uint4& in, float s, uint4& o0, uint4& o1) {
  const uint32_t w[4] = {in.x, in.y, in.z, in.w};
  uint32_t r[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    r[2 * i] = cvt2(static_cast<uint16_t>(w[i] & 0xFFFFu), s);
    r[2 * i + 1] = cvt2(static_cast<uint16_t>(w[i] >> 16), s);
  }
  o0 = make_uint4(r[0], r[1], r[2], r[3]);
  o1 = make_uint4(r[4], r[5], r[6], r[7]);
}

__global__ __launch_bounds__(kDqThreads) void dequant_mla_kernel(const uint8_t* __restrict__ cache, int64_t pool,
                                                                 int64_t slot_stride,
                                                                 const int32_t* __restrict__ slots, int64_t n,
                                                                 uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kDqThreads + threadIdx.x) >> 5;
  const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * kDqThreads) >> 5;
  for (int64_t t0 = warp * kMlaUnroll; t0 < n; t0 += n_warps * kMlaUnroll) {
    uint4 q[kMlaUnroll], rope[kMlaUnroll];
    float s[kMlaUnroll];
    bool ok[kMlaUnroll];
#pragma unroll
    for (int u = 0; u < kMlaUnroll; ++u) {
      const int64_t t = t0 + u;
      int64_t src = t < n ? static_cast<int64_t>(__ldg(slots + t)) : -1;
      ok[u] = t < n && src >= 0 && src < pool;
      if (t < n && !ok[u] && lane == 0) atomicOr(&g_hcu_status, HCU_STATUS_BAD_INPUT);
      src = ok[u] ? src : 0;
      const uint8_t* row = cache + src * slot_stride;
      q[u] = ok[u] ? ld_stream(row + 16 * lane) : make_uint4(0, 0, 0, 0);
      s[u] = ok[u] ? __ldg(reinterpret_cast<const float*>(row + 512) + (lane >> 3)) : 0.f;
      rope[u] = (ok[u] && lane < 8) ? ld_stream(row + 528 + 16 * lane) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kMlaUnroll; ++u) {
      if (!ok[u]) continue;
      uint8_t* dst = reinterpret_cast<uint8_t*>(out + (t0 + u) * kMlaOut);
      uint4 o0, o1;
      cvt16(q[u], s[u], o0, o1);
      st_v4(dst + 32 * lane, o0);
      st_v4(dst + 32 * lane + 16, o1);
      if (lane < 8) st_v4(dst + 1024 + 16 * lane, rope[u]);
    }
  }
}

__global__ __launch_bounds__(kDqThreads, 1) void dequant_index_k_kernel(const uint8_t* __restrict__ kv,
                                                                     int64_t n_pages, int64_t page_stride,
                                                                     const int32_t* __restrict__ loc, int64_t n,
                                                                     uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 3;   // token within the 4-token group
  const int part = lane & 7;   // 16-byte chunk of the token
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kDqThreads + threadIdx.x) >> 5;
  const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * kDqThreads) >> 5;
  const int64_t n_slots = n_pages * kPage;
  for (int64_t t0 = warp * 4 * kIdxUnroll; t0 < n; t0 += n_warps * 4 * kIdxUnroll) {
    uint4 q[kIdxUnroll];
    float s[kIdxUnroll];
    bool ok[kIdxUnroll];
#pragma unroll
    for (int u = 0; u < kIdxUnroll; ++u) {
      const int64_t t = t0 + 4 * u + sub;
      int64_t l = t < n ? static_cast<int64_t>(__ldg(loc + t)) : -1;
      ok[u] = t < n && l >= 0 && l < n_slots;
      if (t < n && !ok[u] && part == 0) atomicOr(&g_hcu_status, HCU_STATUS_BAD_INPUT);
      l = ok[u] ? l : 0;
      const uint8_t* page = kv + (l >> 6) * page_stride;
      q[u] = ok[u] ? ld_stream(page + (l & 63) * kHeadDim + 16 * part) : make_uint4(0, 0, 0, 0);
      s[u] = ok[u] ? __ldg(reinterpret_cast<const float*>(page + kPageFp8Bytes) + (l & 63)) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kIdxUnroll; ++u) {
      if (!ok[u]) continue;
      const int64_t t = t0 + 4 * u + sub;
      uint8_t* dst = reinterpret_cast<uint8_t*>(out + t * kHeadDim);
      uint4 o0, o1;
      cvt16(q[u], s[u], o0, o1);
      st_v4(dst + 32 * part, o0);
      st_v4(dst + 32 * part + 16, o1);
    }
  }
}


// The 16 values of one K row that a lane quantises, held as the raw words loaded (bf16: 8 words,
// two values each; fp32: 16 words) and widened to fp32 on use (bf16 -> fp32 is exact: the bf16
// bits are the high half of the fp32 word).
template <bool kBf16>
struct Row16 {
  static constexpr int kWords = kBf16 ? 8 : 16;
  uint32_t w[kWords];
  __device__ __forceinline__ void load(const void* p) {
#pragma unroll
    for (int i = 0; i < kWords / 4; ++i) {
      const uint4 a = ld_stream(static_cast<const uint8_t*>(p) + 16 * i);
      w[4 * i] = a.x;
      w[4 * i + 1] = a.y;
      w[4 * i + 2] = a.z;
      w[4 * i + 3] = a.w;
    }
  }
  __device__ __forceinline__ float operator[](int j) const {
    if constexpr (kBf16) return __uint_as_float((j & 1) ? (w[j >> 1] & 0xFFFF0000u) : (w[j >> 1] << 16));
    return __uint_as_float(w[j]);
  }
};

// x / s rounded to nearest even, as the fp8 conversion needs it, from rc = RN(1/s) (one correctly
// rounded reciprocal per token instead of 16 divisions per lane): q = RN(x * rc) is within one ulp
// of x / s, the remainder x - q * s is exact in one FMA, and RN(q + rem * rc) is the correctly
// rounded quotient (Markstein's correction theorem: P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990; also
// Muller et al., Handbook of Floating-Point Arithmetic, ch. 4) while the quotient is a normal
// number.  Below 2^-11 the fp8 e4m3 conversion gives a zero of the quotient's sign whatever the
// low bits, and q already has that sign, so q is used there (this also covers s = inf: rc = 0).
// Bit-identical to IEEE division followed by the fp8 conversion (tested against the oracle's
// numpy division, fp8 rounding midpoints included).
__device__ __forceinline__ float div_rn_by(float x, float s, float rc) {
  const float q = x * rc;
  const float rem = fmaf(-q, s, x);
  const float q2 = fmaf(rem, rc, q);
  return fabsf(q) < 0x1p-11f ? q : q2;
}

template <bool kBf16>
__global__ __launch_bounds__(kDqThreads) void quant_store_index_k_kernel(const void* __restrict__ k,
                                                                         int64_t k_stride_bytes,
                                                                         const int32_t* __restrict__ loc, int64_t n,
                                                                         uint8_t* __restrict__ kv, int64_t n_pages,
                                                                         int64_t page_stride) {
  constexpr int kElem = kBf16 ? 2 : 4;
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 3;   // token within the 4-token group
  const int part = lane & 7;   // 16-value chunk of the token
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kDqThreads + threadIdx.x) >> 5;
  const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * kDqThreads) >> 5;
  const int64_t n_slots = n_pages * kPage;
  for (int64_t t0 = warp * 4 * kIdxUnroll; t0 < n; t0 += n_warps * 4 * kIdxUnroll) {
    Row16<kBf16> v[kIdxUnroll];
    int64_t l[kIdxUnroll];
#pragma unroll
    for (int u = 0; u < kIdxUnroll; ++u) {
      const int64_t t = t0 + 4 * u + sub;
      const int64_t tt = t < n ? t : n - 1;  // a full 4-token group of loads; the stores check t
      l[u] = t < n ? static_cast<int64_t>(__ldg(loc + t)) : -1;
      v[u].load(static_cast<const uint8_t*>(k) + tt * k_stride_bytes + 16 * kElem * part);
    }
#pragma unroll
    for (int u = 0; u < kIdxUnroll; ++u) {
      const int64_t t = t0 + 4 * u + sub;
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[u][j]));
      // the 8 lanes of this token (xor 1, 2, 4 stays inside the 8-lane group)
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      const float scale = __fdiv_rn(fmaxf(amax, 1e-12f), 448.f);
      const float rc = __frcp_rn(scale);
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_fp8x2_storage_t lo2 = __nv_cvt_float2_to_fp8x2(
            make_float2(div_rn_by(v[u][4 * i], scale, rc), div_rn_by(v[u][4 * i + 1], scale, rc)), __NV_SATFINITE,
            __NV_E4M3);
        const __nv_fp8x2_storage_t hi2 = __nv_cvt_float2_to_fp8x2(
            make_float2(div_rn_by(v[u][4 * i + 2], scale, rc), div_rn_by(v[u][4 * i + 3], scale, rc)),
            __NV_SATFINITE, __NV_E4M3);
        w[i] = static_cast<uint32_t>(lo2) | (static_cast<uint32_t>(hi2) << 16);
      }
      if (t >= n) continue;
      const bool ok = l[u] >= 0 && l[u] < n_slots;
      if (!ok) {
        if (part == 0) atomicOr(&g_hcu_status, HCU_STATUS_BAD_INPUT);
        continue;
      }
      uint8_t* page = kv + (l[u] >> 6) * page_stride;
      st_v4(page + (l[u] & 63) * kHeadDim + 16 * part, make_uint4(w[0], w[1], w[2], w[3]));
      if (part == 0) reinterpret_cast<float*>(page + kPageFp8Bytes)[l[u] & 63] = scale;
    }
  }
}

// Blocks for `warps_needed` warps of work, at most cap_per_sm per SM (the kernels loop over the
// rest).  The indexer-K dequant runs best at 3 per SM over a grid-stride loop (measured on config 3:
// 12.0 us against 13.1 with every block its own warp's work at 5 resident per SM).
int grid_for(int64_t warps_needed, int cap_per_sm = 8) {
  const int64_t per_block = kDqThreads / 32;
  int64_t blocks = (warps_needed + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * cap_per_sm;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

}  // namespace
}  // namespace hcu

extern "C" int hcu_dequant_k_cache_paged(const uint8_t* quant_k_cache, int64_t pool_slots, int64_t slot_stride,
                                         const int32_t* page_table_1, int64_t n_tokens, uint16_t* out,
                                         hcu_stream_t stream) {
  using namespace hcu;
  if (n_tokens < 0 || pool_slots < 0 || slot_stride < kMlaSlot || slot_stride % 16 != 0) return HCU_ERR_ARG;
  if (n_tokens == 0) return HCU_OK;
  if (!quant_k_cache || !page_table_1 || !out) return HCU_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(quant_k_cache) | reinterpret_cast<uintptr_t>(out)) % 16 != 0)
    return HCU_ERR_ARG;
  const int grid = grid_for((n_tokens + kMlaUnroll - 1) / kMlaUnroll);
  dequant_mla_kernel<<<grid, kDqThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      quant_k_cache, pool_slots, slot_stride, page_table_1, n_tokens, out);
  return launch_status();
}

extern "C" int hcu_dequant_index_k_paged(const uint8_t* kv_cache, int64_t n_pages, int64_t page_stride,
                                         const int32_t* token_loc, int64_t n_tokens, uint16_t* out,
                                         hcu_stream_t stream) {
  using namespace hcu;
  if (n_tokens < 0 || n_pages < 0 || page_stride < kPage * (kHeadDim + 4) || page_stride % 16 != 0)
    return HCU_ERR_ARG;
  if (n_tokens == 0) return HCU_OK;
  if (!kv_cache || !token_loc || !out) return HCU_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(kv_cache) | reinterpret_cast<uintptr_t>(out)) % 16 != 0) return HCU_ERR_ARG;
  const int grid = grid_for((n_tokens + 4 * kIdxUnroll - 1) / (4 * kIdxUnroll), 3);
  dequant_index_k_kernel<<<grid, kDqThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      kv_cache, n_pages, page_stride, token_loc, n_tokens, out);
  return launch_status();
}

extern "C" int hcu_quant_store_index_k_paged(const void* k, int32_t k_dtype, int64_t k_stride,
                                             const int32_t* token_loc, int64_t n_tokens, uint8_t* kv_cache,
                                             int64_t n_pages, int64_t page_stride, hcu_stream_t stream) {
  using namespace hcu;
  if (k_dtype != HCU_DTYPE_F32 && k_dtype != HCU_DTYPE_BF16) return HCU_ERR_ARG;
  const int64_t elem = k_dtype == HCU_DTYPE_BF16 ? 2 : 4;
  if (n_tokens < 0 || n_pages < 0 || k_stride < kHeadDim || (k_stride * elem) % 16 != 0 ||
      page_stride < kPage * (kHeadDim + 4) || page_stride % 16 != 0)
    return HCU_ERR_ARG;
  if (n_tokens == 0) return HCU_OK;
  if (!k || !token_loc || !kv_cache) return HCU_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(kv_cache)) % 16 != 0) return HCU_ERR_ARG;
  const int grid = grid_for((n_tokens + 4 * kIdxUnroll - 1) / (4 * kIdxUnroll));
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (k_dtype == HCU_DTYPE_BF16)
    quant_store_index_k_kernel<true><<<grid, kDqThreads, 0, st>>>(k, k_stride * elem, token_loc, n_tokens, kv_cache,
                                                                  n_pages, page_stride);
  else
    quant_store_index_k_kernel<false><<<grid, kDqThreads, 0, st>>>(k, k_stride * elem, token_loc, n_tokens, kv_cache,
                                                                   n_pages, page_stride);
  return launch_status();
}
