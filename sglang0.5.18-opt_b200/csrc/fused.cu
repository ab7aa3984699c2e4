// Fused prefill indexer: ragged logits -> exact top-2048 without the logits
// round trip through HBM.
//
// The unfused pair writes every (row, token) logit (config 2: 8192 rows x
// ~69K tokens = 2.3 GB) and the top-k reads it back.  Here:
//   1. prep: every kSampleStride-th 128-token tile of K is copied into a small
//      sample K (1/64 of the tokens) and each row's visible sample length is
//      derived from its end;
//   2. the ragged logits kernel scores the rows against the sample K
//      (~1.6 % of the work) and fused_bound_kernel turns each row's sampled
//      scores into a lower estimate of its top-2048 threshold (the sample key
//      of rank t + 5 sqrt(t) + 5, t the threshold's expected sample rank);
//   3. the ragged logits kernel scores the rows against all of K and, instead
//      of storing logits and mask, appends every visible token whose key is at
//      or above the row's estimate to the row's candidate list;
//   4. a select kernel takes the top-2048 of each list and writes it in the
//      canonical order (fused_select_kernel, topk.cu).
// Exactness: every token at or above the estimate is in the list, so when the
// list holds at least 2048 tokens (and did not overflow) the row's threshold is
// at or above the estimate and the list contains the whole top-2048; the keys
// are the ones the top-k derives from the materialised logits (same epilogue
// arithmetic).  A row that fails raises a device flag, and two launches
// predicated on it (the materialising logits kernel, then the top-k over its
// output) rewrite every row: the result never rests on the estimate, and with
// the flag clear those launches return at once (no host synchronisation, so
// the call can be captured in a CUDA graph).
//
// Rows see tokens [0, row_end[r]) (prefix-causal prefill).  The reference has
// no counterpart: its prefill indexer is the closed lightop _mqa_logits
// followed by the materialised top-k (the pair hcu_mqa_logits_ragged +
// hcu_sparse_mask_topk_transform here, whose result this equals).
#include <algorithm>
#include <cstdint>

#include "common.cuh"

namespace hcu {
int launch_ragged_logits(const uint8_t* q, int64_t rows, int64_t heads, const uint8_t* k_fp8, const float* k_scale,
                         int64_t n_tokens, const float* weights, const int32_t* row_start, const int32_t* row_end,
                         float* logits, int64_t logits_stride, int16_t* mask, const int32_t* bounds,
                         int32_t* cand_cnt, int2* cand, int cand_cap, int cand_all_len, const int32_t* run_if,
                         cudaStream_t st);
int launch_fused_select(const int2* cand, const int32_t* cnt, int cap, const int32_t* row_end, int64_t rows,
                        int64_t width, const int32_t* bounds, int all_len, const int32_t* pt, int64_t pt_stride,
                        int32_t* dst, int32_t* flag, cudaStream_t stream);
int launch_topk_if(const float* score, int64_t rows, int64_t width, int64_t score_stride, const int16_t* mask,
                   int64_t mask_stride, const int32_t* lengths, const int32_t* pt, int64_t pt_stride, int32_t* dst,
                   const int32_t* run_if, cudaStream_t stream);
int launch_fused_bound(const float* score, int64_t score_stride, const int16_t* mask, int64_t mask_stride,
                       const int32_t* e_s, const int32_t* row_end, int64_t width, int64_t rows, int32_t* bounds,
                       cudaStream_t stream);
int fused_max_width();
int fused_max_cap();

namespace {

constexpr int kTile = 128;          // K tile of the logits kernels (tokens)
constexpr int kSampleStride = 64;   // one sampled tile in every 64
constexpr int kSampleOffset = 32;   // ... at this position within its group of 64
constexpr int kCandCap = 8192;      // candidate list slots per row
constexpr int kAllLen = 8192;       // rows of at most this many visible tokens list every visible token

struct Layout {
  int64_t n_s_tiles, n_s, s_stride, width_stride;
  int64_t ks_fp8, ks_scale, e_s, zeros, bounds, cnt, flag, lg_s, mk_s, cand, lg, mk, total;
};

int64_t al256(int64_t x) { return (x + 255) / 256 * 256; }

Layout layout(int64_t rows, int64_t n_tokens) {
  Layout L{};
  const int64_t tiles = (n_tokens + kTile - 1) / kTile;
  L.n_s_tiles = tiles > kSampleOffset ? (tiles - kSampleOffset + kSampleStride - 1) / kSampleStride : 0;
  L.n_s = L.n_s_tiles * kTile;
  L.s_stride = (L.n_s + 63) / 64 * 64;
  L.width_stride = (n_tokens + 63) / 64 * 64;
  int64_t o = 0;
  auto take = [&](int64_t bytes) {
    const int64_t at = o;
    o += al256(bytes);
    return at;
  };
  L.ks_fp8 = take(L.n_s * kHeadDim);
  L.ks_scale = take(L.n_s * 4);
  L.e_s = take(rows * 4);
  L.zeros = take(rows * 4);
  L.bounds = take(rows * 4);
  L.cnt = take(rows * 4);
  L.flag = take(4);
  L.lg_s = take(rows * L.s_stride * 4);
  L.mk_s = take(rows * (L.s_stride / 16) * 2);
  L.cand = take(rows * kCandCap * 8);
  L.lg = take(rows * L.width_stride * 4);  // the exact path's logits (written only when the flag is set)
  L.mk = take(rows * (L.width_stride / 16) * 2);
  L.total = o;
  return L;
}

// Blocks [0, n_s_tiles): copy sampled tile j (K tile j * kSampleStride + kSampleOffset; tokens past
// n_tokens as zeros).  Blocks after: per row its visible sample length, a zero row start and a zero
// candidate count; the first of them clears the flag.
__global__ __launch_bounds__(256) void fused_prep_kernel(const uint8_t* __restrict__ k_fp8,
                                                         const float* __restrict__ k_scale, int n_tokens,
                                                         int n_s_tiles, uint8_t* __restrict__ ks_fp8,
                                                         float* __restrict__ ks_scale,
                                                         const int32_t* __restrict__ row_end, int rows,
                                                         int32_t* __restrict__ e_s, int32_t* __restrict__ zeros,
                                                         int32_t* __restrict__ cnt, int32_t* __restrict__ flag) {
  const int b = blockIdx.x;
  if (b < n_s_tiles) {
    const int64_t t0 = (static_cast<int64_t>(b) * kSampleStride + kSampleOffset) * kTile;
    const int valid = static_cast<int>(n_tokens - t0 < kTile ? n_tokens - t0 : kTile);  // >= 1 by the tile count
    const int4* src = reinterpret_cast<const int4*>(k_fp8 + t0 * kHeadDim);
    int4* dst = reinterpret_cast<int4*>(ks_fp8 + static_cast<int64_t>(b) * kTile * kHeadDim);
    for (int i = threadIdx.x; i < kTile * kHeadDim / 16; i += blockDim.x)
      dst[i] = (i >> 3) < valid ? __ldg(src + i) : make_int4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < kTile; i += blockDim.x)
      ks_scale[static_cast<int64_t>(b) * kTile + i] = i < valid ? __ldg(k_scale + t0 + i) : 0.f;
    return;
  }
  const int rb = b - n_s_tiles;
  if (rb == 0 && threadIdx.x == 0) *flag = 0;
  for (int r = rb * blockDim.x + threadIdx.x; r < rows; r += (gridDim.x - n_s_tiles) * blockDim.x) {
    int e = __ldg(row_end + r);
    e = e < 0 ? 0 : (e > n_tokens ? n_tokens : e);
    int64_t seen = 0;
    for (int j = 0; j < n_s_tiles; ++j) {
      const int64_t t0 = (static_cast<int64_t>(j) * kSampleStride + kSampleOffset) * kTile;
      if (t0 >= e) break;
      seen += e - t0 < kTile ? e - t0 : kTile;
    }
    e_s[r] = static_cast<int32_t>(seen);
    zeros[r] = 0;
    cnt[r] = 0;
  }
}

}  // namespace
}  // namespace hcu

extern "C" int64_t hcu_mqa_topk_ragged_workspace_bytes(int64_t rows, int64_t n_tokens) {
  if (rows < 0 || n_tokens < 0) return -1;
  return hcu::layout(rows, n_tokens).total;
}

extern "C" int hcu_mqa_topk_ragged(const uint8_t* q, int64_t rows, int64_t heads, const uint8_t* k_fp8,
                                   const float* k_scale, int64_t n_tokens, const float* weights,
                                   const int32_t* row_end, const int32_t* page_table, int64_t pt_stride,
                                   int32_t* dst, void* workspace, int64_t workspace_bytes, int32_t* fallback_flag,
                                   hcu_stream_t stream) {
  using namespace hcu;
  if (heads != 32 && heads != 64) return HCU_ERR_UNSUPPORTED;
  if (rows < 0 || n_tokens < 0 || rows * heads > INT32_MAX || n_tokens > fused_max_width()) return HCU_ERR_ARG;
  if (rows == 0) return HCU_OK;
  if (!q || !k_fp8 || !k_scale || !weights || !row_end || !page_table || !dst || !workspace || pt_stride < 0)
    return HCU_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_fp8) | reinterpret_cast<uintptr_t>(k_scale) |
       reinterpret_cast<uintptr_t>(weights) | reinterpret_cast<uintptr_t>(workspace)) % 16 != 0)
    return HCU_ERR_ARG;
  const Layout L = layout(rows, n_tokens);
  if (workspace_bytes < L.total) return HCU_ERR_ARG;
  static_assert(kCandCap <= 8192, "list fits the select's shared candidate area");
  if (kCandCap > fused_max_cap()) return HCU_ERR_ARG;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto at = [&](int64_t off) { return ws + off; };
  uint8_t* ks_fp8 = at(L.ks_fp8);
  float* ks_scale = reinterpret_cast<float*>(at(L.ks_scale));
  int32_t* e_s = reinterpret_cast<int32_t*>(at(L.e_s));
  int32_t* zeros = reinterpret_cast<int32_t*>(at(L.zeros));
  int32_t* bounds = reinterpret_cast<int32_t*>(at(L.bounds));
  int32_t* cnt = reinterpret_cast<int32_t*>(at(L.cnt));
  int32_t* flag = reinterpret_cast<int32_t*>(at(L.flag));
  float* lg_s = reinterpret_cast<float*>(at(L.lg_s));
  int16_t* mk_s = reinterpret_cast<int16_t*>(at(L.mk_s));
  int2* cand = reinterpret_cast<int2*>(at(L.cand));
  float* lg = reinterpret_cast<float*>(at(L.lg));
  int16_t* mk = reinterpret_cast<int16_t*>(at(L.mk));

  // 1. sample K, sample lengths, zero row starts, counts and flag
  const int row_blocks = static_cast<int>(std::min<int64_t>((rows + 255) / 256, 1024));
  fused_prep_kernel<<<static_cast<unsigned>(L.n_s_tiles + row_blocks), 256, 0, st>>>(
      k_fp8, k_scale, static_cast<int>(n_tokens), static_cast<int>(L.n_s_tiles), ks_fp8, ks_scale, row_end,
      static_cast<int>(rows), e_s, zeros, cnt, flag);
  int s = launch_status();
  if (s != HCU_OK) return s;
  // 2. sampled scores and the per-row bound (rows without samples get the largest key: their
  //    lists stay empty unless they are short enough to list every token)
  if (L.n_s > 0) {
    if (cudaMemsetAsync(mk_s, 0, static_cast<size_t>(rows * (L.s_stride / 16)) * 2, st) != cudaSuccess)
      return launch_status();
    s = launch_ragged_logits(q, rows, heads, ks_fp8, ks_scale, L.n_s, weights, zeros, e_s, lg_s, L.s_stride, mk_s,
                             nullptr, nullptr, nullptr, 0, 0, nullptr, st);
    if (s != HCU_OK) return s;
    s = launch_fused_bound(lg_s, L.s_stride, mk_s, L.s_stride / 16, e_s, row_end, n_tokens, rows, bounds, st);
  } else {
    s = cudaMemsetAsync(bounds, 0xFF, static_cast<size_t>(rows) * 4, st) == cudaSuccess ? HCU_OK : launch_status();
  }
  if (s != HCU_OK) return s;
  // 3. full scores into the candidate lists
  s = launch_ragged_logits(q, rows, heads, k_fp8, k_scale, n_tokens, weights, zeros, row_end, nullptr,
                           L.width_stride, nullptr, bounds, cnt, cand, kCandCap, kAllLen, nullptr, st);
  if (s != HCU_OK) return s;
  // 4. select + canonical order; rows that fail raise the flag
  s = launch_fused_select(cand, cnt, kCandCap, row_end, rows, n_tokens, bounds, kAllLen, page_table, pt_stride, dst,
                          flag, st);
  if (s != HCU_OK) return s;
  // exact path, predicated on the flag: materialised logits (every mask word below a row's end is
  // written by the kernel itself, rows starting at 0), then the top-k of every row
  s = launch_ragged_logits(q, rows, heads, k_fp8, k_scale, n_tokens, weights, zeros, row_end, lg, L.width_stride, mk,
                           nullptr, nullptr, nullptr, 0, 0, flag, st);
  if (s != HCU_OK) return s;
  s = launch_topk_if(lg, rows, n_tokens, L.width_stride, mk, L.width_stride / 16, row_end, page_table, pt_stride, dst,
                     flag, st);
  if (s != HCU_OK) return s;
  if (fallback_flag &&
      cudaMemcpyAsync(fallback_flag, flag, sizeof(int32_t), cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return launch_status();
  return HCU_OK;
}
