// Stage 2: MQA index logits on the 5th-generation tensor cores (sm_100a).
//
//   s[row, t] = (sum_h w[row, h] * relu(q[row, h, :] . k[t, :])) * k_scale[t]
//
// Paged decode kernel (mqa_logits_paged_kernel), one persistent CTA per SM:
//   * the work list is (request group, row block, 128-token tile) flattened in
//     that order and cut into one contiguous range per CTA (balanced to one
//     tile; Q changes only at group boundaries).  It is derived on the device
//     from the context lengths, so the launch is CUDA-graph capturable;
//   * warp 0 (TMA producer): per tile two 3-D TMA box loads {128 B, 64 tok, 1}
//     of the two 64-token K pages named by the block table (128-byte swizzle,
//     a K-major UMMA operand), into an 8-stage ring; per group the R*H Q rows
//     (2-D TMA) into a double buffer;
//   * warp 1 (MMA issuer): tcgen05.mma.cta_group::1.kind::f8f6f4, M = 128
//     tokens, N = R*H query heads, K = 128 as 4 x 32, accumulating fp32 in a
//     double-buffered TMEM accumulator; tcgen05.commit frees the stage and
//     publishes the accumulator;
//   * warps 2-5 (epilogue): thread = token = TMEM lane; tcgen05.ld of the row's
//     H columns, ReLU * w head sum in registers, * k_scale, mask bit via warp
//     ballot, logits stored only where the bit is set.
// Semantics follow hcu_ops/csrc/mqa_hist.cu:97-273 of the reference: lengths
// clamped to [0, width], every row of a group reads the group's first block
// table row, mask bit = token < len && bits(s) != 0.
//
// Every mbarrier wait is bounded (common.cuh); on expiry the CTA records
// HCU_STATUS_WAIT_TIMEOUT, stops issuing, drains the copies and MMAs it issued
// and frees its TMEM before returning.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

HCU_DEFINE_STATUS(status_logits)

namespace hcu {
int launch_pass1_hist(const float* logits, int64_t rows, int64_t width, const int16_t* mask, int64_t mask_stride,
                      const int32_t* hist_lens, int32_t* zws, cudaStream_t stream);

namespace {

constexpr int kLgThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpiWarps = 8;
constexpr int kMaxAcc = 4;     // TMEM accumulator buffers (4 when N <= 128, else 2)
constexpr int kStages = 8;
constexpr int kTileTok = 128;
constexpr int kATile = kTileTok * kHeadDim;  // 16 KB
constexpr int kMaxN = 256;
constexpr int kQTile = kMaxN * kHeadDim;  // 32 KB

constexpr int kBtWin = 256;  // block-table entries staged in shared memory by the producer warp

struct __align__(1024) LgSmem {
  uint8_t a[kStages][kATile];      // K tile: two 64-token pages, 128-byte swizzled rows
  uint8_t q[2][kQTile];            // Q rows of the current row block (double buffered)
  float sc[kStages][2 * kPage];    // k_scale of the stage's two pages
  float w[kEpiWarps][kMaxN];       // head weights, one copy per epilogue warp
  int lens[kEpiWarps][8];          // row lengths of the current row block, per epilogue warp
  int bt[kBtWin];                  // producer's window of the current group's block-table row
  uint64_t full[kStages];
  uint64_t empty[kStages];         // 1 MMA commit + 8 epilogue warps (they read sc[] after the MMA)
  uint64_t qfull[2];
  uint64_t qempty[2];
  uint64_t tfull[kMaxAcc];
  uint64_t tempty[kMaxAcc];
  uint64_t done;
  uint32_t tmem_base;
  int start_group;
  int start_local;
  int count;
  int abort;
};

struct PagedArgs {
  const uint8_t* kv;
  int64_t page_stride;
  int64_t n_pages;
  const float* weights;
  const int32_t* ctx_lens;
  const int32_t* bt;
  int64_t bt_stride;
  float* logits;
  int16_t* mask;
  int batch;
  int G;       // rows per request group (share the first row's block table)
  int R;       // rows per CTA row block (R * H <= 256)
  int width;   // logits row width = block-table capacity * 64
};

__device__ __forceinline__ int clamp_len(int l, int width) { return l < 0 ? 0 : (l > width ? width : l); }

__device__ __forceinline__ int group_len(const PagedArgs& p, int g) {
  int m = 0;
  for (int r = 0; r < p.G; ++r) m = max(m, clamp_len(__ldg(p.ctx_lens + g * p.G + r), p.width));
  return m;
}

__device__ __forceinline__ int group_tiles(const PagedArgs& p, int g) {
  return (group_len(p, g) + kTileTok - 1) / kTileTok;
}

// Cursor over this CTA's contiguous range of (group, row block, tile) items.
struct Cursor {
  int g, li, len, tiles, n_sub;
  __device__ void init(const PagedArgs& p, int g0, int l0) {
    g = g0;
    li = l0;
    n_sub = (p.G + p.R - 1) / p.R;
    len = group_len(p, g);
    tiles = (len + kTileTok - 1) / kTileTok;
  }
  // Advances to the next item; returns (sub, tile) of the current one.
  __device__ void next(const PagedArgs& p, int& sub, int& tile) {
    while (li >= tiles * n_sub) {
      ++g;
      li = 0;
      len = group_len(p, g);
      tiles = (len + kTileTok - 1) / kTileTok;
    }
    sub = li / tiles;
    tile = li - sub * tiles;
    ++li;
  }
};

template <int H>
__global__ __launch_bounds__(kLgThreads, 1) void mqa_logits_paged_kernel(const __grid_constant__ CUtensorMap tm_kv,
                                                                        const __grid_constant__ CUtensorMap tm_sc,
                                                                        const __grid_constant__ CUtensorMap tm_q,
                                                                        const PagedArgs p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  LgSmem& sm = *reinterpret_cast<LgSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_groups = p.batch / p.G;
  const int n_sub = (p.G + p.R - 1) / p.R;
  const int NC = p.R * H;  // TMEM columns per accumulator buffer
  const int NACC = NC <= 128 ? 4 : 2;

  // ---- schedule: this CTA's contiguous item range (warp 0, all lanes) ----
  if (warp == 0) {
    int64_t total = 0;
    for (int base = 0; base < n_groups; base += 32) {
      const int g = base + lane;
      int c = g < n_groups ? group_tiles(p, g) * n_sub : 0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
      total += c;
    }
    const int64_t begin = total * blockIdx.x / gridDim.x;
    const int64_t end = total * (blockIdx.x + 1) / gridDim.x;
    int sg = 0, sl = 0;
    if (end > begin) {
      int64_t run = 0;
      for (int base = 0; base < n_groups; base += 32) {
        const int g = base + lane;
        const int c = g < n_groups ? group_tiles(p, g) * n_sub : 0;
        int inc = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, inc, o);
          if (lane >= o) inc += y;
        }
        const bool hit = run + inc > begin && c > 0;
        const uint32_t bal = __ballot_sync(0xffffffffu, hit);
        if (bal) {
          const int src = __ffs(bal) - 1;
          const int inc_s = __shfl_sync(0xffffffffu, inc, src);
          const int c_s = __shfl_sync(0xffffffffu, c, src);
          sg = base + src;
          sl = static_cast<int>(begin - (run + inc_s - c_s));
          break;
        }
        run += __shfl_sync(0xffffffffu, inc, 31);
      }
    }
    if (lane == 0) {
      sm.start_group = sg;
      sm.start_local = sl;
      sm.count = static_cast<int>(end - begin);
    }
  }
  __syncthreads();
  const int count = sm.count;
  if (count <= 0) return;  // uniform: before any barrier init or TMEM allocation

  uint32_t ncols = 32;
  while (ncols < static_cast<uint32_t>(NACC * NC)) ncols <<= 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1 + kEpiWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.qfull[i], 1);
      mbar_init(&sm.qempty[i], 1);
    }
    for (int i = 0; i < kMaxAcc; ++i) {
      mbar_init(&sm.tfull[i], 1);
      mbar_init(&sm.tempty[i], kEpiWarps);
    }
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_kv);
    tma_prefetch_desc(&tm_sc);
    tma_prefetch_desc(&tm_q);
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem_base, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (whole warp; lane 0 issues)
    Cursor cur;
    cur.init(p, sm.start_group, sm.start_local);
    int qkey = -1, qn = 0, issued = 0;
    int win_g = -1, win_base = 0;
    for (int it = 0; it < count; ++it) {
      int sub, tile;
      cur.next(p, sub, tile);
      const int n_pg = (cur.len + kPage - 1) / kPage;
      const int p0 = 2 * tile;
      const bool two = p0 + 1 < n_pg;
      if (cur.g != win_g || p0 < win_base || p0 + 1 >= win_base + kBtWin) {
        // stage the next kBtWin block-table entries of this group with one coalesced warp load
        __syncwarp();
        win_g = cur.g;
        win_base = p0;
        const int32_t* btr = p.bt + static_cast<int64_t>(cur.g) * p.G * p.bt_stride;
        for (int i = lane; i < kBtWin; i += 32) {
          const int pg = win_base + i;
          sm.bt[i] = pg < n_pg ? __ldg(btr + pg) : 0;
        }
        __syncwarp();
      }
      const int ph0 = sm.bt[p0 - win_base];
      const int ph1 = two ? sm.bt[p0 + 1 - win_base] : 0;
      int ok = 1;
      if (lane == 0) {
        const int key = cur.g * n_sub + sub;
        if (key != qkey) {
          const int j = qn;
          ok = mbar_wait(&sm.qempty[j & 1], ((j >> 1) & 1) ^ 1, abort, &g_hcu_status);
          if (ok) {
            mbar_arrive_expect_tx(&sm.qfull[j & 1], static_cast<uint32_t>(NC * kHeadDim));
            tma_load_2d(sm.q[j & 1], &tm_q, &sm.qfull[j & 1], 0, (cur.g * p.G + sub * p.R) * H);
            ++qn;
            qkey = key;
          }
        }
        const int s = it % kStages;
        if (ok) ok = mbar_wait(&sm.empty[s], ((it / kStages) & 1) ^ 1, abort, &g_hcu_status);
        if (ok) {
          const uint32_t bytes = (two ? 2u : 1u) * (kPageFp8Bytes + kPage * 4);
          mbar_arrive_expect_tx(&sm.full[s], bytes);
          tma_load_3d(sm.a[s], &tm_kv, &sm.full[s], 0, 0, ph0);
          tma_load_2d(sm.sc[s], &tm_sc, &sm.full[s], 0, ph0);
          if (two) {
            tma_load_3d(sm.a[s] + kPageFp8Bytes, &tm_kv, &sm.full[s], 0, 0, ph1);
            tma_load_2d(sm.sc[s] + kPage, &tm_sc, &sm.full[s], 0, ph1);
          }
          issued = it + 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    }
    if (lane == 0) {
      // Drain: every copy issued must land before the CTA may exit.
      const int first = issued > kStages ? issued - kStages : 0;
      for (int it = first; it < issued; ++it)
        mbar_wait_drain(&sm.full[it % kStages], (it / kStages) & 1, &g_hcu_status);
      for (int j = qn > 2 ? qn - 2 : 0; j < qn; ++j) mbar_wait_drain(&sm.qfull[j & 1], (j >> 1) & 1, &g_hcu_status);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (elect_one()) {
      Cursor cur;
      cur.init(p, sm.start_group, sm.start_local);
      int qkey = -1;
      int qn = 0;
      uint32_t idesc = 0;
      for (int it = 0; it < count; ++it) {
        int sub, tile;
        cur.next(p, sub, tile);
        const int key = cur.g * n_sub + sub;
        if (key != qkey) {
          if (qn > 0) tc_commit(&sm.qempty[(qn - 1) & 1]);
          const int j = qn;
          if (!mbar_wait(&sm.qfull[j & 1], (j >> 1) & 1, abort, &g_hcu_status)) break;
          ++qn;
          qkey = key;
          const int nr = min(p.R, p.G - sub * p.R);
          idesc = idesc_e4m3_f32(128, nr * H);
        }
        const int s = it % kStages;
        const int a = it % NACC;
        if (!mbar_wait(&sm.full[s], (it / kStages) & 1, abort, &g_hcu_status)) break;
        if (!mbar_wait(&sm.tempty[a], ((it / NACC) & 1) ^ 1, abort, &g_hcu_status)) break;
        tc_fence_after();
        const uint64_t adesc = sw128_kmajor_desc(smem_u32(sm.a[s]));
        const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sm.q[(qn - 1) & 1]));
        const uint32_t d = tmem + static_cast<uint32_t>(a * NC);
#pragma unroll
        for (int k = 0; k < kHeadDim / 32; ++k)
          mma_f8f6f4(d, adesc + 2 * k, bdesc + 2 * k, idesc, k > 0 ? 1u : 0u);
        tc_commit(&sm.empty[s]);
        tc_commit(&sm.tfull[a]);
      }
      tc_commit(&sm.done);
      mbar_wait_drain(&sm.done, 0, &g_hcu_status);
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..9)
    // Two warps per TMEM lane quadrant: with >= 2 rows per block they split the
    // rows (r % 2 == half); a single-row block alternates tiles between them.
    const int ew = warp - 2;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int half = ew >> 2;
    float* wsm = sm.w[ew];
    int* lsm = sm.lens[ew];
    Cursor cur;
    cur.init(p, sm.start_group, sm.start_local);
    int qkey = -1;
    int nr = 0;
    const int64_t mstride = p.width / 16;
    for (int it = 0; it < count; ++it) {
      int sub, tile;
      cur.next(p, sub, tile);
      const int key = cur.g * n_sub + sub;
      const int row0 = cur.g * p.G + sub * p.R;
      if (key != qkey) {
        nr = min(p.R, p.G - sub * p.R);
        __syncwarp();
        for (int i = lane; i < nr * H; i += 32) wsm[i] = __ldg(p.weights + static_cast<int64_t>(row0) * H + i);
        if (lane < nr) lsm[lane] = clamp_len(__ldg(p.ctx_lens + row0 + lane), p.width);
        __syncwarp();
        qkey = key;
      }
      const int tok_in_tile = quad * 32 + lane;
      const int tok_base = tile * kTileTok + quad * 32;
      const int token = tok_base + lane;
      const int s = it % kStages;
      const int a = it % NACC;
      if (!mbar_wait(&sm.tfull[a], (it / NACC) & 1, abort, &g_hcu_status)) break;
      tc_fence_after();
      const float ksc = sm.sc[s][tok_in_tile];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[s]);  // this warp is done with the stage's scales
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(a * NC);
      const int r_first = nr >= 2 ? half : ((it & 1) == half ? 0 : nr);
      const int r_step = nr >= 2 ? 2 : 1;
      for (int r = r_first; r < nr; r += r_step) {
        uint32_t v[H / 32][32];
#pragma unroll
        for (int c = 0; c < H / 32; ++c) tmem_ld_x32(tbase + r * H + c * 32, v[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < H / 32; ++c) tmem_reg_fence(v[c]);
        // 8 independent chains: 4 packed fp32 pairs
        float2 acc0 = make_float2(0.f, 0.f), acc1 = acc0, acc2 = acc0, acc3 = acc0;
#pragma unroll
        for (int c = 0; c < H / 32; ++c) {
          const float4* w4 = reinterpret_cast<const float4*>(wsm + r * H + c * 32);
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const float4 wa = w4[j];
            const float4 wb = w4[j + 1];
            const uint32_t* x = &v[c][4 * j];
            acc0 = fma2(make_float2(fmaxf(__uint_as_float(x[0]), 0.f), fmaxf(__uint_as_float(x[1]), 0.f)),
                        make_float2(wa.x, wa.y), acc0);
            acc1 = fma2(make_float2(fmaxf(__uint_as_float(x[2]), 0.f), fmaxf(__uint_as_float(x[3]), 0.f)),
                        make_float2(wa.z, wa.w), acc1);
            acc2 = fma2(make_float2(fmaxf(__uint_as_float(x[4]), 0.f), fmaxf(__uint_as_float(x[5]), 0.f)),
                        make_float2(wb.x, wb.y), acc2);
            acc3 = fma2(make_float2(fmaxf(__uint_as_float(x[6]), 0.f), fmaxf(__uint_as_float(x[7]), 0.f)),
                        make_float2(wb.z, wb.w), acc3);
          }
        }
        float s0 = ((acc0.x + acc0.y) + (acc1.x + acc1.y)) + ((acc2.x + acc2.y) + (acc3.x + acc3.y));
        s0 *= ksc;
        const int row = row0 + r;
        const bool keep = token < lsm[r] && __float_as_uint(s0) != 0u;
        const uint32_t bits = __ballot_sync(0xffffffffu, keep);
        if (lane == 0 && tok_base < p.width)
          reinterpret_cast<uint32_t*>(p.mask)[(static_cast<int64_t>(row) * mstride + tok_base / 16) >> 1] = bits;
        if (keep) p.logits[static_cast<int64_t>(row) * p.width + token] = s0;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.tempty[a]);
    }
  }

  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

bool make_map_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_pages(CUtensorMap* m, const void* base, uint64_t n_pages, uint64_t page_stride) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(kPage), n_pages};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadDim), page_stride};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kHeadDim), static_cast<cuuint32_t>(kPage), 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// k_scale rows of the pages: 64 fp32 at byte 8192 of each page.
bool make_map_page_scales(CUtensorMap* m, const uint8_t* kv, uint64_t n_pages, uint64_t page_stride) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kPage), n_pages};
  cuuint64_t strides[1] = {page_stride};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kPage), 1};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<uint8_t*>(kv + kPageFp8Bytes), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int H>
int launch_paged(const CUtensorMap& tkv, const CUtensorMap& tsc, const CUtensorMap& tq, const PagedArgs& a,
                 cudaStream_t stream) {
  const size_t smem = sizeof(LgSmem) + 1024;
  cudaFuncSetAttribute(mqa_logits_paged_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  mqa_logits_paged_kernel<H><<<sm_count(), kLgThreads, smem, stream>>>(tkv, tsc, tq, a);
  return launch_status();
}

}  // namespace
}  // namespace hcu

extern "C" int hcu_mqa_logits_hist(const uint8_t* q, int64_t batch, int64_t heads, const uint8_t* kv_cache,
                                   int64_t n_pages, int64_t page_stride, const float* weights,
                                   const int32_t* context_lens, const int32_t* block_table, int64_t bt_stride,
                                   int64_t max_context_len, int64_t group_size, int64_t persistent_ctas,
                                   int64_t rows_per_cta, const int32_t* hist_lens, float* logits, int16_t* mask,
                                   int32_t* zws, hcu_stream_t stream) {
  using namespace hcu;
  (void)persistent_ctas;  // scheduling is derived from the SM count and the lengths on the device
  if (heads != 32 && heads != 64) return HCU_ERR_UNSUPPORTED;
  if (batch <= 0 || group_size <= 0 || batch % group_size != 0 || batch * heads > INT32_MAX) return HCU_ERR_ARG;
  if (max_context_len <= 0 || max_context_len % kPage != 0 || max_context_len > (1ll << 30)) return HCU_ERR_ARG;
  if (bt_stride < max_context_len / kPage || n_pages <= 0 || n_pages > INT32_MAX) return HCU_ERR_ARG;
  if (page_stride < kPage * (kHeadDim + 4) || page_stride % 16 != 0) return HCU_ERR_ARG;
  if (!q || !kv_cache || !weights || !context_lens || !block_table || !logits || !mask) return HCU_ERR_ARG;
  if (hist_lens && !zws) return HCU_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kv_cache) | reinterpret_cast<uintptr_t>(mask) |
       reinterpret_cast<uintptr_t>(weights)) % 16 != 0)
    return HCU_ERR_ARG;
  int64_t R = std::min<int64_t>(group_size, kMaxN / heads);
  if (rows_per_cta > 0 && rows_per_cta < R) R = rows_per_cta;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t mask_words = max_context_len / 16;
  if (cudaMemsetAsync(mask, 0, static_cast<size_t>(batch * mask_words) * sizeof(int16_t), st) != cudaSuccess)
    return launch_status();
  CUtensorMap tkv, tsc, tq;
  if (!make_map_pages(&tkv, kv_cache, static_cast<uint64_t>(n_pages), static_cast<uint64_t>(page_stride)))
    return HCU_ERR_LAUNCH;
  if (!make_map_page_scales(&tsc, kv_cache, static_cast<uint64_t>(n_pages), static_cast<uint64_t>(page_stride)))
    return HCU_ERR_LAUNCH;
  if (!make_map_2d(&tq, q, kHeadDim, static_cast<uint64_t>(batch * heads), kHeadDim, kHeadDim,
                   static_cast<uint32_t>(R * heads), CU_TENSOR_MAP_SWIZZLE_128B))
    return HCU_ERR_LAUNCH;
  PagedArgs a;
  a.kv = kv_cache;
  a.page_stride = page_stride;
  a.n_pages = n_pages;
  a.weights = weights;
  a.ctx_lens = context_lens;
  a.bt = block_table;
  a.bt_stride = bt_stride;
  a.logits = logits;
  a.mask = mask;
  a.batch = static_cast<int>(batch);
  a.G = static_cast<int>(group_size);
  a.R = static_cast<int>(R);
  a.width = static_cast<int>(max_context_len);
  int stt = heads == 64 ? launch_paged<64>(tkv, tsc, tq, a, st) : launch_paged<32>(tkv, tsc, tq, a, st);
  if (stt != HCU_OK) return stt;
  if (hist_lens) return launch_pass1_hist(logits, batch, max_context_len, mask, mask_words, hist_lens, zws, st);
  return HCU_OK;
}

extern "C" int hcu_mqa_logits_ragged(const uint8_t* q, int64_t rows, int64_t heads, const uint8_t* k_fp8,
                                     const float* k_scale, int64_t n_tokens, const float* weights,
                                     const int32_t* row_start, const int32_t* row_end, float* logits,
                                     int64_t logits_stride, int16_t* mask, hcu_stream_t stream) {
  (void)q; (void)rows; (void)heads; (void)k_fp8; (void)k_scale; (void)n_tokens; (void)weights;
  (void)row_start; (void)row_end; (void)logits; (void)logits_stride; (void)mask; (void)stream;
  return HCU_ERR_UNSUPPORTED;
}
