// Context-parallel merge: P per-range top-2048 lists -> the global top-2048.
//
// Rank p of a KV-range split owns the contiguous global token range
// [p*N/P, (p+1)*N/P) and emits (uint32 key, global index) for its local
// top-2048 in ascending token order (hcu_topk_keys).  Concatenating the lists
// in rank order therefore lists every candidate in ascending global index, and
// the global top-2048 under (key desc, index asc) is a subset of the union.
// One 1024-thread CTA per row: a 12/12/8-bit radix select finds the threshold
// key, then an ordered compaction writes the keys above it in index order
// followed by the first `remaining` ties in index order -- the canonical order
// of the single-GPU top-k, so the CP result equals the 1-GPU result exactly.
// Rows whose total visible length is at most 2048 keep every candidate in
// index order (decided by the length, not the candidate count: one range may
// hold all of a longer row's top-k).
#include "common.cuh"

HCU_DEFINE_STATUS(status_merge)

namespace hcu {
namespace {

constexpr int kMgThreads = 1024;
constexpr int kMgWarps = kMgThreads / 32;
constexpr int kMaxParts = 16;

struct MergeSmem {
  int hist[kBins + 32];
  int wtot[kMgWarps];
  int wtot2[kMgWarps];
  int res[4];
};

// Exclusive block scan of two non-negative counters; returns totals.
__device__ __forceinline__ void block_scan2(int a, int b, int& ea, int& eb, int& ta, int& tb, int* wa, int* wb) {
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  int ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ya = __shfl_up_sync(0xffffffffu, ia, o);
    const int yb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += ya;
      ib += yb;
    }
  }
  if (lane == 31) {
    wa[w] = ia;
    wb[w] = ib;
  }
  __syncthreads();
  int pa = 0, pb = 0, sa = 0, sb = 0;
  for (int v = 0; v < kMgWarps; ++v) {
    const int x = wa[v], y = wb[v];
    pa += v < w ? x : 0;
    pb += v < w ? y : 0;
    sa += x;
    sb += y;
  }
  __syncthreads();
  ea = pa + ia - a;
  eb = pb + ib - b;
  ta = sa;
  tb = sb;
}

template <int NB>
__device__ __forceinline__ void find_thr(const int* hist, int need, int* wtot, int* res) {
  constexpr int BPT = NB >= kMgThreads ? NB / kMgThreads : 1;
  constexpr int ACTIVE = NB / BPT;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int w = tid >> 5;
  int h[BPT];
  int s = 0;
#pragma unroll
  for (int j = 0; j < BPT; ++j) {
    h[j] = tid < ACTIVE ? hist[tid * BPT + j] : 0;
    s += h[j];
  }
  int x = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_down_sync(0xffffffffu, x, o);
    if (lane + o < 32) x += y;
  }
  if (lane == 0) wtot[w] = x;
  __syncthreads();
  int after = 0;
  for (int v = w + 1; v < kMgWarps; ++v) after += wtot[v];
  const int suf = x + after;
  const int suf_next = suf - s;
  if (tid < ACTIVE && suf >= need && suf_next < need) {
    int acc = suf_next;
#pragma unroll
    for (int j = BPT - 1; j >= 0; --j) {
      if (acc + h[j] >= need) {
        res[0] = tid * BPT + j;
        res[1] = acc;
        break;
      }
      acc += h[j];
    }
  }
  __syncthreads();
}

// Thread t owns candidates [t*per, (t+1)*per) of the concatenated list
// (candidate c = part c / 2048, slot c % 2048).
__global__ __launch_bounds__(kMgThreads, 1) void cp_merge_kernel(const uint32_t* __restrict__ keys,
                                                                const int32_t* __restrict__ gidx, int parts,
                                                                int rows, const int32_t* __restrict__ lengths,
                                                                int32_t* __restrict__ dst) {
  __shared__ MergeSmem sm;
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int per = parts * kTopK / kMgThreads;  // parts * 2 candidates per thread
  const int c0 = tid * per;
  auto cand = [&](int c, uint32_t& k, int& g) {
    const int64_t off = (static_cast<int64_t>(c / kTopK) * rows + row) * kTopK + (c % kTopK);
    k = __ldg(keys + off);
    g = __ldg(gidx + off);
  };
  int32_t* out = dst + static_cast<int64_t>(row) * kTopK;

  int nvalid = 0;
  for (int i = 0; i < per; ++i) {
    uint32_t k;
    int g;
    cand(c0 + i, k, g);
    nvalid += g >= 0;
  }
  int ev, dummy, total, dummy2;
  block_scan2(nvalid, 0, ev, dummy, total, dummy2, sm.wtot, sm.wtot2);
  if (__ldg(lengths + row) <= kTopK) {
    int pos = ev;
    for (int i = 0; i < per; ++i) {
      uint32_t k;
      int g;
      cand(c0 + i, k, g);
      if (g >= 0 && pos < kTopK) out[pos++] = g;
    }
    for (int i = min(total, kTopK) + tid; i < kTopK; i += kMgThreads) out[i] = -1;
    return;
  }
  if (total < kTopK) {  // inconsistent lengths: keep what there is, in index order
    if (tid == 0) atomicOr(&g_hcu_status, HCU_STATUS_BAD_INPUT);
    int pos = ev;
    for (int i = 0; i < per; ++i) {
      uint32_t k;
      int g;
      cand(c0 + i, k, g);
      if (g >= 0) out[pos++] = g;
    }
    for (int i = total + tid; i < kTopK; i += kMgThreads) out[i] = -1;
    return;
  }

  // pass 1: key[31:20]
  for (int i = tid; i < kBins; i += kMgThreads) sm.hist[i] = 0;
  __syncthreads();
  for (int i = 0; i < per; ++i) {
    uint32_t k;
    int g;
    cand(c0 + i, k, g);
    if (g >= 0) atomicAdd(&sm.hist[k >> 20], 1);
  }
  __syncthreads();
  find_thr<kBins>(sm.hist, kTopK, sm.wtot, sm.res);
  const uint32_t t1 = static_cast<uint32_t>(sm.res[0]);
  const int need1 = kTopK - sm.res[1];
  // pass 2: key[19:8] inside t1
  for (int i = tid; i < kBins; i += kMgThreads) sm.hist[i] = 0;
  __syncthreads();
  for (int i = 0; i < per; ++i) {
    uint32_t k;
    int g;
    cand(c0 + i, k, g);
    if (g >= 0 && (k >> 20) == t1) atomicAdd(&sm.hist[(k >> 8) & 0xFFFu], 1);
  }
  __syncthreads();
  find_thr<kBins>(sm.hist, need1, sm.wtot, sm.res);
  const uint32_t p24 = (t1 << 12) | static_cast<uint32_t>(sm.res[0]);
  const int need2 = need1 - sm.res[1];
  // pass 3: key[7:0] inside p24
  for (int i = tid; i < 256; i += kMgThreads) sm.hist[i] = 0;
  __syncthreads();
  for (int i = 0; i < per; ++i) {
    uint32_t k;
    int g;
    cand(c0 + i, k, g);
    if (g >= 0 && (k >> 8) == p24) atomicAdd(&sm.hist[k & 0xFFu], 1);
  }
  __syncthreads();
  find_thr<256>(sm.hist, need2, sm.wtot, sm.res);
  const uint32_t thr = (p24 << 8) | static_cast<uint32_t>(sm.res[0]);
  const int remaining = need2 - sm.res[1];
  const int tie_base = kTopK - remaining;

  int na = 0, nt = 0;
  for (int i = 0; i < per; ++i) {
    uint32_t k;
    int g;
    cand(c0 + i, k, g);
    na += (g >= 0) & (k > thr);
    nt += (g >= 0) & (k == thr);
  }
  int ea, et, ta, tt;
  block_scan2(na, nt, ea, et, ta, tt, sm.wtot, sm.wtot2);
  for (int i = 0; i < per; ++i) {
    uint32_t k;
    int g;
    cand(c0 + i, k, g);
    if (g < 0) continue;
    if (k > thr) {
      out[ea++] = g;
    } else if (k == thr) {
      if (et < remaining) out[tie_base + et] = g;
      ++et;
    }
  }
}

}  // namespace
}  // namespace hcu

extern "C" int hcu_cp_topk_merge(const uint32_t* keys, const int32_t* gidx, int64_t n_parts, int64_t rows,
                                 const int32_t* lengths, int32_t* dst, hcu_stream_t stream) {
  using namespace hcu;
  if (n_parts < 1 || n_parts > kMaxParts || rows < 0 || rows > INT32_MAX) return HCU_ERR_ARG;
  if (rows == 0) return HCU_OK;
  if (!keys || !gidx || !lengths || !dst) return HCU_ERR_ARG;
  // per-thread candidate count must be integral: parts * 2048 divisible by 1024
  cp_merge_kernel<<<static_cast<unsigned>(rows), kMgThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      keys, gidx, static_cast<int>(n_parts), static_cast<int>(rows), lengths, dst);
  return launch_status();
}
