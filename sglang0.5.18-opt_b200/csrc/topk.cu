// Stage 3: exact top-2048 over masked scores + page-table transform.
//
// topk_row_kernel: one CTA (1024 or 512 threads) per row.
// Candidate path (the normal case, one streaming pass over the row):
//   S  m strided samples (2048 for rows <= 128K tokens) go into a 12-bit and
//      then an 8-bit histogram; the sample order statistic a few sigma below
//      the threshold's expected sample rank gives a lower bound lo (20 key
//      bits resolved).  With the logits kernel's exact pass-1 histogram (the
//      "pre" path) lo is the threshold's 12-bit bin instead, with no sampling.
//   P  rounds of 16384 tokens (lane: 16 consecutive tokens; warp: 512): every
//      token with key >= lo is appended to a shared-memory candidate list at
//      its block-wide prefix position, so the list is in token order.  For a
//      positive lo the test is one signed compare of the raw float bits.
//   Q  a 9-bit-digit radix select over the candidates (digits below the
//      common prefix of lo and the largest candidate) gives the threshold key,
//      the count above it and the number of ties to take.
//   R  one block scan of (above, tie) flags over the list writes the output.
// Exact fallback, when the list holds fewer than 2048 tokens (the bound
// missed) or more than its capacity (heavy ties, a sparse row whose threshold
// is +0); the row stays L2-resident:
//   X  the threshold key by a descent over four 8-bit key digits, most
//      significant first: per level one streaming pass builds per-warp digit
//      histograms of the keys that share the digits found so far (the +0 key
//      of unset mask bits counted in registers), and a rank search over their
//      sum picks the next digit;
//   Y  one streaming pass in block-wide rounds writes the selection in order:
//      a block scan of each thread's (above, tie) counts gives every selected
//      token its output position directly.
// Unset mask bits are an implicit +0 (key 0x80000000) whatever the score
// storage holds.  The selection and output order are those of
// hcu_ops/csrc/sparse_mask_topk.cu:1-7,141-349 of the reference: keys larger
// than the threshold in token order, then the first threshold ties in token
// order (ties broken toward the lower index).
#include <cooperative_groups.h>
#include <cstddef>

#include <mutex>
#include <vector>

#include "common.cuh"

HCU_DEFINE_STATUS(status_topk)

namespace hcu {
namespace {

constexpr int kSmallSample = 2048;  // row samples used to bound the threshold (rows <= 128K)
constexpr int kSample = 8192;       // sample count for rows > 512K
constexpr int kLaneTok = 16;        // consecutive tokens per lane in a streaming round
constexpr int kNarrowWidth = 32768; // rows up to this width run the 512-thread kernel (two CTAs per SM)
constexpr int kManyRowsWidth = 98304;  // ... and up to this width when the rows fill the SMs twice over
constexpr int kMaxClusterSplits = 8;  // CTAs per row of a split row (portable cluster size)
constexpr int kSplitMinTok = 8192;    // a split row gives each CTA at least this many visible tokens

// Per-CTA-size constants: 1024 threads (one CTA per SM) for wide rows, 512 threads for
// narrow ones (and for rows up to 96K tokens when there are at least two rows per SM), so
// that two CTAs per SM overlap their rows' latency-bound phases.
template <int kT>
struct Tk {
  static constexpr int kWarps = kT / 32;
  static constexpr int kRound = kT * kLaneTok;               // tokens per streaming round
  static constexpr int kCandCap = kT >= 1024 ? 8192 : 4096;  // candidate list capacity
  static constexpr int kMaxSample = kT >= 1024 ? kSample : kSmallSample;
  // sampled bound: one kBins histogram; exact fallback: per-warp 256-bin digit histograms + their sum
  static constexpr int kHist = kWarps * 256 + 256 > kBins ? kWarps * 256 + 256 : kBins;
};

template <int kT>
struct __align__(16) TopkSmem {
  int hist[Tk<kT>::kHist];  // sampled bound: [0, 4096); fallback: warps x 256 digit counts, then their sum
  uint4 scr[kLaneTok / 4][kT];  // candidate pass: this thread's current 16 score words
  uint32_t cand_key[Tk<kT>::kCandCap];
  int32_t cand_idx[Tk<kT>::kCandCap];
  int32_t cand_pid[Tk<kT>::kCandCap];  // page-table entry of each candidate (async copies)
  alignas(16) int hb[2][512];  // digit histograms (sample refinement: 256 bins, candidate select: 512); read as int4
  int wcnt[2][Tk<kT>::kWarps];
  uint32_t wmax[Tk<kT>::kWarps];
  int above[Tk<kT>::kWarps];
  int ties[Tk<kT>::kWarps];
  int zeros[Tk<kT>::kWarps];
  int pos[Tk<kT>::kWarps];
  int wtot[32];
  int res[4];
  int ncand;  // split rows: this CTA's candidate count (read by the cluster's rank 0)
  int mark_any;        // CP merge: some list of the row was truncated (marker entry -2)
  uint32_t mark_max;   // CP merge: the largest marker key
};

// 4-byte global -> shared copy that does not hold a register (LDGSTS).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ int warp_sum(int x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Branch-free monotone key.
__device__ __forceinline__ uint32_t key_of(float x) {
  const uint32_t b = __float_as_uint(x);
  return b ^ (static_cast<uint32_t>(static_cast<int32_t>(b) >> 31) | 0x80000000u);
}

// Loads the 16 consecutive tokens [i0, i0 + 16) (i0 % 16 == 0) of this lane:
// their keys (unset mask bit -> +0) and the mask of slots below `lim`.
template <bool kVec>
__device__ __forceinline__ uint32_t load16(const float* __restrict__ vals, const int16_t* __restrict__ mrow, int i0,
                                           int lim, uint32_t (&k)[16]) {
  if (i0 >= lim) {
#pragma unroll
    for (int t = 0; t < 16; ++t) k[t] = kZeroKey;
    return 0u;
  }
  const uint32_t mw = static_cast<uint16_t>(__ldg(mrow + (i0 >> 4)));
  float v[16];
  if constexpr (kVec) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i0 + 4 * q < lim) f = __ldg(reinterpret_cast<const float4*>(vals + i0 + 4 * q));
      v[4 * q] = f.x;
      v[4 * q + 1] = f.y;
      v[4 * q + 2] = f.z;
      v[4 * q + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int t = 0; t < 16; ++t) v[t] = i0 + t < lim ? __ldg(vals + i0 + t) : 0.f;
  }
#pragma unroll
  for (int t = 0; t < 16; ++t) k[t] = ((mw >> t) & 1u) ? key_of(v[t]) : kZeroKey;
  const int nv = lim - i0;
  return nv >= 16 ? 0xFFFFu : ((1u << nv) - 1u);
}

__device__ __forceinline__ int warp_incl_scan(int x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

// Warp 0 of the block: bin b of the NB-bin histogram h with
// suffix(b) >= need > suffix(b+1); res[0] = b, res[1] = suffix(b+1).
// Requires sum(h) >= need >= 1.
template <int NB>
__device__ __forceinline__ void warp_find(const int* h, int need, int* res) {
  constexpr int P = NB / 32;  // bins per lane
  const int lane = threadIdx.x & 31;
  int v[P];
#pragma unroll
  for (int q = 0; q < P / 4; ++q) {
    const int4 a = reinterpret_cast<const int4*>(h)[lane * (P / 4) + q];
    v[4 * q] = a.x;
    v[4 * q + 1] = a.y;
    v[4 * q + 2] = a.z;
    v[4 * q + 3] = a.w;
  }
  int s = 0;
#pragma unroll
  for (int j = 0; j < P; ++j) s += v[j];
  int x = s;  // inclusive suffix over lanes >= lane
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_down_sync(0xffffffffu, x, o);
    if (lane + o < 32) x += y;
  }
  const int nxt = x - s;
  if (x >= need && nxt < need) {
    int acc = nxt;
#pragma unroll
    for (int j = P - 1; j >= 0; --j) {
      if (acc + v[j] >= need) {
        res[0] = lane * P + j;
        res[1] = acc;
        break;
      }
      acc += v[j];
    }
  }
}

// Exclusive block-wide prefix sum of x; *total = the block sum.  One barrier;
// consecutive calls must be separated by a barrier (wtot is reused).
template <int kT>
__device__ __forceinline__ int block_excl_scan(int x, int* wtot, int* total) {
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int inc = warp_incl_scan(x);
  if (lane == 31) wtot[w] = inc;
  __syncthreads();
  const int t = lane < kT / 32 ? wtot[lane] : 0;
  const int ti = warp_incl_scan(t);
  *total = __shfl_sync(0xffffffffu, ti, 31);
  return __shfl_sync(0xffffffffu, ti - t, w) + inc - x;
}

// Rank search over an NB-bin histogram h (shared or global memory): the bin b
// holding the need-th largest key, i.e. S(b) >= need > S(b + 1) with S(b) the
// count in bins >= b; res[0] = b, res[1] = S(b + 1).  Requires sum(h) >= need
// >= 1.  Thread t takes the t-th run of NB / kT bins counted down from the top
// bin, so an exclusive block scan of the run totals in thread order is the
// count above each run.  Called by every thread after a barrier that published
// h; ends with a barrier (res is then visible to all).
template <int kT, int NB>
__device__ __forceinline__ void block_rank_bin(const int* h, int need, int* wtot, int* res) {
  constexpr int kRun = NB >= kT ? NB / kT : 1;
  constexpr int kRuns = NB / kRun;
  const int t = threadIdx.x;
  const int top = NB - 1 - t * kRun;  // highest bin of this thread's run
  int c[kRun];
  int s = 0;
#pragma unroll
  for (int j = 0; j < kRun; ++j) {
    c[j] = t < kRuns ? h[top - j] : 0;
    s += c[j];
  }
  int total;
  int acc = block_excl_scan<kT>(s, wtot, &total);  // keys in the runs above this one
  if (t < kRuns && acc < need && acc + s >= need) {
#pragma unroll
    for (int j = 0; j < kRun; ++j) {
      if (acc + c[j] >= need) {
        res[0] = top - j;
        res[1] = acc;
        break;
      }
      acc += c[j];
    }
  }
  __syncthreads();
}

// Raw float bits of this lane's 16 consecutive tokens [i0, i0 + 16) (0 at and
// past `lim`); `valid` = the slots below lim.  Returns their mask word.
template <bool kVec>
__device__ __forceinline__ uint32_t load16_raw(const float* __restrict__ vals, const int16_t* __restrict__ mrow,
                                               int i0, int lim, uint32_t (&b)[16], uint32_t& valid) {
  if (i0 >= lim) {
#pragma unroll
    for (int t = 0; t < 16; ++t) b[t] = 0u;
    valid = 0u;
    return 0u;
  }
  const uint32_t mw = static_cast<uint16_t>(__ldg(mrow + (i0 >> 4)));
  if constexpr (kVec) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 f = make_uint4(0u, 0u, 0u, 0u);
      if (i0 + 4 * q < lim) f = __ldg(reinterpret_cast<const uint4*>(vals + i0 + 4 * q));
      b[4 * q] = f.x;
      b[4 * q + 1] = f.y;
      b[4 * q + 2] = f.z;
      b[4 * q + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int t = 0; t < 16; ++t) b[t] = i0 + t < lim ? __float_as_uint(__ldg(vals + i0 + t)) : 0u;
  }
  const int nv = lim - i0;
  valid = nv >= 16 ? 0xFFFFu : ((1u << nv) - 1u);
  return mw;
}

// One round of the candidate pass for the 16 tokens of this lane whose raw
// bits are in X (round r).  The words go to this thread's scratch slot, X is
// refilled with round r + 2, and after the round's barrier the candidates are
// appended at their block-wide prefix position, visiting set bits only.
template <int kT, bool kVec, bool kPos>
__device__ __forceinline__ void candidate_round(const float* __restrict__ vals, const int16_t* __restrict__ mrow,
                                                const int32_t* __restrict__ src, int seg0, int len, uint32_t lo, int r,
                                                int nr,
                                                TopkSmem<kT>& sm,
                                                uint32_t (&X)[16], uint32_t& mX, uint32_t& vX, int& base,
                                                uint32_t& kmax) {
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int i0 = seg0 + r * Tk<kT>::kRound + w * (32 * kLaneTok) + lane * kLaneTok;
  const int lim_pos = static_cast<int>(lo ^ kZeroKey);
  uint32_t cb = 0u;
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    bool c;
    if constexpr (kPos) {
      c = static_cast<int>(X[t]) >= lim_pos;
    } else {
      c = (((mX >> t) & 1u) ? key_of(__uint_as_float(X[t])) : kZeroKey) >= lo;
    }
    cb |= static_cast<uint32_t>(c) << t;
  }
  cb &= kPos ? (mX & vX) : vX;
  const uint32_t mcur = mX;
  if (cb) {
#pragma unroll
    for (int q = 0; q < 4; ++q) sm.scr[q][threadIdx.x] = make_uint4(X[4 * q], X[4 * q + 1], X[4 * q + 2], X[4 * q + 3]);
  }
  const int nc = __popc(cb);
  const int inc = warp_incl_scan(nc);
  if (lane == 31) sm.wcnt[r & 1][w] = inc;
  if (r + 2 < nr) mX = load16_raw<kVec>(vals, mrow, i0 + 2 * Tk<kT>::kRound, len, X, vX);
  __syncthreads();
  const int wc = lane < kT / 32 ? sm.wcnt[r & 1][lane] : 0;  // one entry per warp
  const int wi = warp_incl_scan(wc);
  const int wbase = __shfl_sync(0xffffffffu, wi - wc, w);
  const int rtot = __shfl_sync(0xffffffffu, wi, 31);
  int pos = base + wbase + inc - nc;
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(&sm.scr[0][threadIdx.x]);
  while (cb) {
    const int t = __ffs(cb) - 1;
    cb &= cb - 1u;
    const uint32_t raw = mine[(t >> 2) * (4 * kT) + (t & 3)];
    uint32_t key;
    if constexpr (kPos) {
      key = raw | kZeroKey;
    } else {
      key = ((mcur >> t) & 1u) ? key_of(__uint_as_float(raw)) : kZeroKey;
    }
    kmax = key > kmax ? key : kmax;
    if (pos < Tk<kT>::kCandCap) {
      sm.cand_key[pos] = key;
      sm.cand_idx[pos] = i0 + t;
      cp_async4(&sm.cand_pid[pos], src + i0 + t);
    }
    ++pos;
  }
  base += rtot;
}

// Candidate pass: appends every token of [seg0, len) whose key is >= lo to
// sm.cand_key / sm.cand_idx in token order, in block-wide rounds of kRound
// tokens (warp w takes tokens [w*512, w*512+512) of a round, lane l 16 of
// them; rounds start at seg0, a multiple of 16).  A / mA / vA hold round 0's
// loads on entry; two rounds of loads are
// in flight at every barrier.  kPos (lo > +0): a token is a candidate iff its
// mask bit is set and its float bits, as a signed integer, are >=
// lo ^ 0x80000000.  Returns the candidate count (nothing past kCandCap is
// stored); sm.wmax receives each warp's largest candidate key.  Each stored
// candidate's page-table entry src[idx] is copied to sm.cand_pid
// asynchronously (waited for in write_candidates).
template <int kT, bool kVec, bool kPos>
__device__ __forceinline__ int collect_candidates(const float* __restrict__ vals, const int16_t* __restrict__ mrow,
                                                  const int32_t* __restrict__ src, int seg0, int len, uint32_t lo,
                                                  TopkSmem<kT>& sm, uint32_t (&A)[16], uint32_t mA, uint32_t vA) {
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int nr = (len - seg0 + Tk<kT>::kRound - 1) / Tk<kT>::kRound;
  uint32_t B[16], mB = 0u, vB = 0u;
  if (nr > 1)
    mB = load16_raw<kVec>(vals, mrow, seg0 + Tk<kT>::kRound + w * (32 * kLaneTok) + lane * kLaneTok, len, B, vB);
  int base = 0;
  uint32_t kmax = 0u;
  for (int r = 0; r < nr; r += 2) {
    candidate_round<kT, kVec, kPos>(vals, mrow, src, seg0, len, lo, r, nr, sm, A, mA, vA, base, kmax);
    if (r + 1 < nr)
      candidate_round<kT, kVec, kPos>(vals, mrow, src, seg0, len, lo, r + 1, nr, sm, B, mB, vB, base, kmax);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t y = __shfl_xor_sync(0xffffffffu, kmax, o);
    kmax = y > kmax ? y : kmax;
  }
  if (lane == 0) sm.wmax[w] = kmax;
  __syncthreads();
  return base;
}

// Threshold key of rank k (kTopK by default) among the n candidates (k <= n <= kCandCap,
// all keys >= lo): a radix select of u = key - lo with 9-bit digits from the
// top bit of (largest candidate - lo) down.  *above = candidates with a
// larger key.  sm.hb[0] and sm.hb[1] must be zero on entry.
template <int kT, class Sm>
__device__ __forceinline__ uint32_t select_candidates_in(Sm& sm, int n, uint32_t lo, int* above, int k = kTopK);

template <int kT>
__device__ __forceinline__ uint32_t select_candidates(TopkSmem<kT>& sm, int n, uint32_t lo, int* above,
                                                     int k = kTopK) {
  return select_candidates_in<kT>(sm, n, lo, above, k);
}

// The select over any shared-memory layout holding cand_key[], wmax[], hb[2][512] and res[].
template <int kT, class Sm>
__device__ __forceinline__ uint32_t select_candidates_in(Sm& sm, int n, uint32_t lo, int* above, int k) {
  constexpr int kDigit = 9;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int w = tid >> 5;
  uint32_t kmax = lane < kT / 32 ? sm.wmax[lane] : 0u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t y = __shfl_xor_sync(0xffffffffu, kmax, o);
    kmax = y > kmax ? y : kmax;
  }
  const uint32_t span = kmax - lo;
  const int d = span ? 31 - __clz(span) : 0;  // every u has no bit above d
  uint32_t pre = 0u;
  int need = k;
  int abv = 0;
  for (int s = d + 1 - kDigit, rnd = 0;; s -= kDigit, ++rnd) {
    const int sh = s > 0 ? s : 0;
    const int nb = s + kDigit - sh;  // bits in this digit (the last one may be short)
    const uint32_t dm = (1u << nb) - 1u;
    int* h = sm.hb[rnd & 1];
    for (int i = tid; i < n; i += kT) {
      const uint32_t u = sm.cand_key[i] - lo;
      if ((static_cast<uint64_t>(u) >> (sh + nb)) == pre) atomicAdd(&h[(u >> sh) & dm], 1);
    }
    for (int i = tid; i < 512; i += kT) sm.hb[(rnd + 1) & 1][i] = 0;
    __syncthreads();
    if (w == 0) warp_find<512>(h, need, sm.res);
    __syncthreads();
    abv += sm.res[1];
    need -= sm.res[1];
    pre = (pre << nb) | static_cast<uint32_t>(sm.res[0]);
    if (sh == 0) break;
  }
  *above = abv;
  return lo + pre;
}

// Output from the candidate list: keys > thr in token order, then the first
// k - above ties in token order (kSorted: the same set in token order),
// through the page-table entries copied during the candidate pass.
// Candidate i goes to thread i / ceil(n / 1024).
template <int kT, bool kSorted>
__device__ __forceinline__ void write_candidates(TopkSmem<kT>& sm, int n, uint32_t thr, int above,
                                                 int32_t* __restrict__ out, uint32_t* __restrict__ okeys,
                                                 int k = kTopK) {
  const int remaining = k - above;
  const int per = (n + kT - 1) / kT;
  const int i0 = min(n, static_cast<int>(threadIdx.x) * per);
  const int i1 = min(n, i0 + per);
  int na = 0, nt = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t k = sm.cand_key[i];
    na += k > thr;
    nt += k == thr;
  }
  cp_async_wait_all();  // the barrier in the scan publishes every thread's page-id copies
  int total;
  const int ex = block_excl_scan<kT>(na | (nt << 16), sm.wtot, &total);
  int ea = ex & 0xFFFF;
  int et = ex >> 16;
  for (int i = i0; i < i1; ++i) {
    const uint32_t k = sm.cand_key[i];
    int p = -1;
    if (k > thr) {
      p = kSorted ? ea + min(et, remaining) : ea;
      ++ea;
    } else if (k == thr) {
      if (et < remaining) p = kSorted ? ea + et : above + et;
      ++et;
    }
    if (p >= 0) {
      out[p] = sm.cand_pid[i];
      if (okeys) okeys[p] = k;
    }
  }
}

// Cluster gather of a split row, called by every CTA of the cluster after its
// candidate pass (sm.ncand = its count, sm.wmax its warps' maxima).  Rank 0
// appends the lists of ranks 1.. after its own (rank order = token order) by
// distributed shared-memory loads and folds their warp maxima into sm.wmax;
// the second cluster barrier keeps every CTA resident until rank 0 has read
// its list.  Returns the total candidate count on rank 0 (past kCandCap when
// any list or the union overflows), 0 elsewhere.
template <int kT>
__device__ __noinline__ int split_gather(TopkSmem<kT>& sm, int splits, int rank) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  int n = 0;
  if (rank == 0) {
    n = sm.ncand;
    bool over = n > Tk<kT>::kCandCap;
    for (int r = 1; r < splits; ++r) {
      TopkSmem<kT>* rs = cluster.map_shared_rank(&sm, r);
      const int nr = rs->ncand;
      if (nr > Tk<kT>::kCandCap || n + nr > Tk<kT>::kCandCap) over = true;
      if (!over)
        for (int i = threadIdx.x; i < nr; i += kT) {
          sm.cand_key[n + i] = rs->cand_key[i];
          sm.cand_idx[n + i] = rs->cand_idx[i];
          sm.cand_pid[n + i] = rs->cand_pid[i];
        }
      if (threadIdx.x < kT / 32) {
        const uint32_t m = rs->wmax[threadIdx.x];
        if (m > sm.wmax[threadIdx.x]) sm.wmax[threadIdx.x] = m;
      }
      n += nr;
    }
    if (over) n = Tk<kT>::kCandCap + 1;
  }
  cluster.sync();
  return n;
}

// ---------------------------------------------------------------------------
// Exact fallback (X, Y of the header).  A "key source" visits, for the calling
// thread, every valid key it owns: f(key) per key.  The digit descent works
// on any source (row tokens here, exchanged list entries in the CP merge).
// ---------------------------------------------------------------------------

// Row tokens [0, len): thread t owns the 16-token chunks starting at
// 16 (t + k kT) (one 64-byte run per lane, 2 KB per warp and round).
template <int kT, bool kVec>
struct RowKeys {
  const float* vals;
  const int16_t* mrow;
  int len;
  template <class F>
  __device__ __forceinline__ void operator()(F&& f) const {
    for (int i0 = static_cast<int>(threadIdx.x) * kLaneTok; i0 < len; i0 += kT * kLaneTok) {
      uint32_t k[16];
      const uint32_t vm = load16<kVec>(vals, mrow, i0, len, k);
#pragma unroll
      for (int t = 0; t < 16; ++t)
        if ((vm >> t) & 1u) f(k[t]);
    }
  }
};

// The key of rank k (1 = largest) among the source's keys and *above = the
// number of keys strictly larger (the k - *above first ties complete the
// selection).  Requires k <= number of keys.  Four levels of 8-bit digits:
// level L histograms digit L of the keys whose higher digits equal the prefix
// found so far, into one 256-bin histogram per warp (no inter-warp atomics);
// the +0 key, which dominates sparse rows, is counted in registers and added
// once per warp.  Every thread of the CTA calls it.
template <int kT, class Src>
__device__ __noinline__ uint32_t digit_descent(TopkSmem<kT>& sm, const Src& src, int k, int* above) {
  constexpr int kW = kT / 32;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  int* wh = sm.hist + (tid >> 5) * 256;
  int* sum = sm.hist + kW * 256;  // 16-byte aligned (warp_find reads it as int4)
  uint32_t prefix = 0u;
  int need = k;
  int abv = 0;
#pragma unroll 1
  for (int level = 0; level < 4; ++level) {
    const int sh = 24 - 8 * level;
    for (int i = tid; i < kW * 256; i += kT) sm.hist[i] = 0;
    __syncthreads();
    int zc = 0;
    src([&](uint32_t key) {
      if (key == kZeroKey) {
        ++zc;
      } else if (level == 0 || (key >> (sh + 8)) == prefix) {
        atomicAdd(&wh[(key >> sh) & 0xFFu], 1);
      }
    });
    zc = warp_sum(zc);
    if (lane == 0 && zc && (level == 0 || (kZeroKey >> (sh + 8)) == prefix))
      atomicAdd(&wh[(kZeroKey >> sh) & 0xFFu], zc);
    __syncthreads();
    if (tid < 256) {
      int c = 0;
#pragma unroll 4
      for (int v = 0; v < kW; ++v) c += sm.hist[v * 256 + tid];
      sum[tid] = c;
    }
    __syncthreads();
    if ((tid >> 5) == 0) warp_find<256>(sum, need, sm.res);
    __syncthreads();
    prefix = (prefix << 8) | static_cast<uint32_t>(sm.res[0]);
    abv += sm.res[1];
    need -= sm.res[1];
  }
  *above = abv;
  return prefix;
}

// Writes the selection of a row given its threshold: keys > thr, then the
// first `remaining` ties, both in token order (kSorted: the same set in token
// order), through the page table.  Block-wide rounds of kT x 16 tokens; one
// block scan per round of each thread's packed (above, tie) counts (a round
// holds at most 16384 tokens, so 16 bits each suffice) gives each selected
// token its position.  Stops once every output slot is written.
template <int kT, bool kVec, bool kSorted>
__device__ __noinline__ void ordered_write_row(TopkSmem<kT>& sm, const float* __restrict__ vals,
                                               const int16_t* __restrict__ mrow, const int32_t* __restrict__ src,
                                               int len, uint32_t thr, int above, int32_t* __restrict__ out,
                                               uint32_t* __restrict__ okeys) {
  const int remaining = kTopK - above;
  int base_a = 0, base_t = 0;  // above / tie tokens in earlier rounds
  for (int r0 = 0; r0 < len; r0 += kT * kLaneTok) {
    const int i0 = r0 + static_cast<int>(threadIdx.x) * kLaneTok;
    uint32_t k[16];
    const uint32_t vm = load16<kVec>(vals, mrow, i0, len, k);
    uint32_t ab = 0u, tb = 0u;
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      ab |= static_cast<uint32_t>(k[t] > thr) << t;
      tb |= static_cast<uint32_t>(k[t] == thr) << t;
    }
    ab &= vm;
    tb &= vm;
    int total;
    const int ex = block_excl_scan<kT>(__popc(ab) | (__popc(tb) << 16), sm.wtot, &total);
    int pa = base_a + (ex & 0xFFFF);
    int pq = base_t + (ex >> 16);
    if (ab | tb) {
#pragma unroll
      for (int t = 0; t < 16; ++t) {  // static indices: k[] stays in registers
        int p = -1;
        if ((ab >> t) & 1u) {
          p = kSorted ? pa + min(pq, remaining) : pa;
          ++pa;
        } else if ((tb >> t) & 1u) {
          if (pq < remaining) p = kSorted ? pa + pq : above + pq;
          ++pq;
        }
        if (p >= 0) {
          out[p] = __ldg(src + i0 + t);
          if (okeys) okeys[p] = k[t];
        }
      }
    }
    base_a += total & 0xFFFF;
    base_t += total >> 16;
    __syncthreads();  // wtot is reused by the next round's scan
    if (base_a >= above && base_t >= remaining) break;  // block-uniform
  }
}

// kSplit: the row is split over a cluster of `splits` CTAs (blockIdx.x = row *
// splits + rank): each derives the same bound lo over the whole row and
// collects the candidates of its own token range; rank 0 gathers the lists
// from the other CTAs' shared memory (rank order = token order) and selects.
template <int kT, bool kVec, bool kSorted, bool kSplit>
__global__ __launch_bounds__(kT, 1024 / kT) void topk_row_kernel(
    const float* __restrict__ score, int64_t score_stride, int width, const int16_t* __restrict__ mask,
    int64_t mask_stride, const int32_t* __restrict__ lengths, const int32_t* __restrict__ pt, int64_t pt_stride,
    int32_t* __restrict__ dst, uint32_t* __restrict__ dst_keys, const int32_t* __restrict__ pre_ws, int rows,
    int splits, const int32_t* __restrict__ run_if, int run_if_stride) {
  constexpr int kTkThreads = kT;
  constexpr int kCandCap = Tk<kT>::kCandCap;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TopkSmem<kT>& sm = *reinterpret_cast<TopkSmem<kT>*>(smem_raw);
  // launched with programmatic stream serialization: wait for the previous kernel (the logits that
  // this reads) to complete before the first global read; a no-op after an ordinary dependency
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // predicated launch (one word for every row, or a word per row): nothing to do this time
  if (run_if != nullptr &&
      __ldcg(run_if + static_cast<int64_t>(kSplit ? static_cast<int>(blockIdx.x) / splits : blockIdx.x) *
                          run_if_stride) == 0)
    return;
  const int row = kSplit ? static_cast<int>(blockIdx.x) / splits : static_cast<int>(blockIdx.x);
  const int rank = kSplit ? static_cast<int>(blockIdx.x) % splits : 0;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int w = tid >> 5;
  int len = lengths[row];
  len = len < width ? len : width;
  len = len < 0 ? 0 : len;
  const int32_t* src = pt + static_cast<int64_t>(row) * pt_stride;
  int32_t* out = dst + static_cast<int64_t>(row) * kTopK;
  const float* vals = score + static_cast<int64_t>(row) * score_stride;
  const int16_t* mrow = mask + static_cast<int64_t>(row) * mask_stride;

  // split rows: CTAs that share the row (at most one per kSplitMinTok visible tokens); with one,
  // rank 0 runs the plain single-CTA path and the others leave at once
  int s_eff = 1;
  if constexpr (kSplit) {
    s_eff = min(splits, max(1, len / kSplitMinTok));
    if (s_eff == 1 && rank != 0) return;
  }

  if (len <= kTopK) {
    if (rank != 0) return;
    for (int i = tid; i < kTopK; i += kTkThreads) {
      out[i] = i < len ? src[i] : -1;
      if (dst_keys) {
        uint32_t k = 0;
        if (i < len) {
          const bool set = (static_cast<uint16_t>(mrow[i >> 4]) >> (i & 15)) & 1u;
          k = set ? to_key(vals[i]) : kZeroKey;
        }
        dst_keys[static_cast<int64_t>(row) * kTopK + i] = k;
      }
    }
    return;
  }

  // this CTA's token range of the candidate pass (the whole row unless split)
  const int cseg = s_eff > 1 ? (len + s_eff * 512 - 1) / (s_eff * 512) * 512 : len;
  const int cs0 = min(rank * cseg, len);
  const int cs1 = min(cs0 + cseg, len);

  uint32_t* const okeys = dst_keys ? dst_keys + static_cast<int64_t>(row) * kTopK : nullptr;
  {
    // ---- candidate path ----
    // The sample loads go out first (they gate the bound), then round 0's
    // loads, whose latency overlaps the bound search.
    const int m = min(Tk<kT>::kMaxSample, len <= (1 << 17) ? kSmallSample : (len <= (1 << 19) ? 4096 : kSample));
    const int groups = m / 4;  // m samples in groups of 4 consecutive tokens, one 16-byte load each
    constexpr int kGpt = Tk<kT>::kMaxSample / (4 * kTkThreads);  // sample groups per thread (at most)
    float sv[4 * kGpt];
    uint32_t smb[kGpt];
    if (pre_ws == nullptr) {
      const float stride_g = static_cast<float>(len) / static_cast<float>(groups);
      const int gmax = (len - 4) & ~3;
#pragma unroll
      for (int j = 0; j < kGpt; ++j) {
        const int g = tid + j * kTkThreads;
        smb[j] = 0u;
#pragma unroll
        for (int e = 0; e < 4; ++e) sv[4 * j + e] = 0.f;
        if (g < groups) {
          const int i = min(gmax, static_cast<int>((static_cast<float>(g) + 0.5f) * stride_g) & ~3);
          smb[j] = (static_cast<uint16_t>(__ldg(mrow + (i >> 4))) >> (i & 15)) & 0xFu;
          if constexpr (kVec) {
            const float4 f = __ldg(reinterpret_cast<const float4*>(vals + i));
            sv[4 * j] = f.x;
            sv[4 * j + 1] = f.y;
            sv[4 * j + 2] = f.z;
            sv[4 * j + 3] = f.w;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) sv[4 * j + e] = __ldg(vals + i + e);
          }
        }
      }
    }
    uint32_t b0[16], valid0;
    const uint32_t mw0 = load16_raw<kVec>(vals, mrow, cs0 + w * (32 * kLaneTok) + lane * kLaneTok, cs1, b0, valid0);
    for (int i = tid; i < 2 * 512; i += kTkThreads) (&sm.hb[0][0])[i] = 0;
    uint32_t lo = 0u;
    bool try_cand = false;
    if (pre_ws == nullptr) {
      for (int i = tid; i < kBins; i += kTkThreads) sm.hist[i] = 0;
      __syncthreads();
      const float stride_f = static_cast<float>(len) / static_cast<float>(m);
      uint32_t sk[4 * kGpt];
#pragma unroll
      for (int j = 0; j < 4 * kGpt; ++j) {
        sk[j] = ((smb[j / 4] >> (j % 4)) & 1u) ? key_of(sv[j]) : kZeroKey;
        if (tid + (j / 4) * kTkThreads < groups) atomicAdd(&sm.hist[sk[j] >> 20], 1);
      }
      __syncthreads();
      // sample rank (1 = largest) 4 sigma + 4 below the threshold's expected sample rank
      const float t = static_cast<float>(kTopK) / stride_f;
      const int r_lo = min(m, static_cast<int>(ceilf(t + 4.f * sqrtf(t) + 4.f)));
      block_rank_bin<kT, kBins>(sm.hist, r_lo, sm.wtot, sm.res);
      const uint32_t b1 = static_cast<uint32_t>(sm.res[0]);
      const int need = r_lo - sm.res[1];
#pragma unroll
      for (int j = 0; j < 4 * kGpt; ++j)
        if (tid + (j / 4) * kTkThreads < groups && (sk[j] >> 20) == b1)
          atomicAdd(&sm.hb[0][(sk[j] >> 12) & 0xFFu], 1);
      __syncthreads();
      if (w == 0) warp_find<256>(sm.hb[0], need, sm.res);
      __syncthreads();
      lo = (b1 << 20) | (static_cast<uint32_t>(sm.res[0]) << 12);
      if (tid < 256) sm.hb[0][tid] = 0;  // ordered before the select by the candidate pass's barriers
      try_cand = true;
    } else {
      // the logits kernel's exact pass-1 histogram: lo = the threshold's 12-bit bin
      const int* h1 = pre_ws + static_cast<int64_t>(row) * kBins;
      const int* cnt = pre_ws + 2 * static_cast<int64_t>(rows) * kBins + 2 * row;
      const int positives = cnt[0];
      const int zeros = cnt[1];
      if (!(positives <= kTopK && positives + zeros >= kTopK)) {
        if (tid == 0) {  // a histogram that does not hold kTopK tokens leaves lo = 0 (still exact)
          sm.res[0] = 0;
          sm.res[1] = 0;
        }
        __syncthreads();  // res written above before the search (and wtot free)
        block_rank_bin<kT, kBins>(h1, kTopK, sm.wtot, sm.res);
        const int b1 = sm.res[0];
        lo = static_cast<uint32_t>(b1) << 20;
        try_cand = sm.res[1] + h1[b1] <= kCandCap;
      }
    }
    if (kSplit && s_eff > 1) {
      // every CTA of the cluster reaches both cluster barriers (s_eff and try_cand are the same for all of them)
      int n = 0;
      if (try_cand) {
        const int nl = lo > kZeroKey ? collect_candidates<kT, kVec, true>(vals, mrow, src, cs0, cs1, lo, sm, b0, mw0, valid0)
                                     : collect_candidates<kT, kVec, false>(vals, mrow, src, cs0, cs1, lo, sm, b0, mw0, valid0);
        cp_async_wait_all();  // this CTA's page ids are in its shared memory before the gather
        if (tid == 0) sm.ncand = nl;
        n = split_gather(sm, splits, rank);
      }
      if (rank != 0) return;
      if (try_cand && n >= kTopK && n <= kCandCap) {
        int above = 0;
        const uint32_t thr = select_candidates(sm, n, lo, &above);
        write_candidates<kT, kSorted>(sm, n, thr, above, out, okeys);
        return;
      }
      try_cand = false;  // rank 0 alone runs the exact fallback over the whole row
    }
    if (try_cand) {
      const int n = lo > kZeroKey ? collect_candidates<kT, kVec, true>(vals, mrow, src, 0, len, lo, sm, b0, mw0, valid0)
                                  : collect_candidates<kT, kVec, false>(vals, mrow, src, 0, len, lo, sm, b0, mw0, valid0);
      if (n < kTopK || n > kCandCap) cp_async_wait_all();  // no copy outlives the candidate path
      if (n >= kTopK && n <= kCandCap) {
        int above = 0;
        const uint32_t thr = select_candidates(sm, n, lo, &above);
        write_candidates<kT, kSorted>(sm, n, thr, above, out, okeys);
        return;
      }
    }
    __syncthreads();
  }

  // ---- exact fallback: threshold by digit descent, then the ordered write ----
  int above = 0;
  const uint32_t thr = digit_descent(sm, RowKeys<kT, kVec>{vals, mrow, len}, kTopK, &above);
  ordered_write_row<kT, kVec, kSorted>(sm, vals, mrow, src, len, thr, above, out, okeys);
}

// ---------------------------------------------------------------------------
// Pass 1 as its own kernels (used by hcu_mqa_logits_hist when hist_lens is
// given): workspace zws = [ghist1 rows*4096 | ghist2 rows*4096 | cnt rows*2],
// the contract of hcu_ops/csrc/mqa_hist.cu:219-226,253-303 of the reference.
// ---------------------------------------------------------------------------
constexpr int kHistThreads = 512;
constexpr int kHistChunk = 16384;

__global__ __launch_bounds__(256) void hist_init_kernel(int32_t* __restrict__ zws, const int32_t* __restrict__ hist_lens,
                                                       int width, int rows) {
  const int row = blockIdx.x;
  int h = hist_lens[row];
  h = h < width ? h : width;
  const int zeros = h > kTopK ? h : 0;
  int4* g1 = reinterpret_cast<int4*>(zws + static_cast<int64_t>(row) * kBins);
  int4* g2 = reinterpret_cast<int4*>(zws + static_cast<int64_t>(rows + row) * kBins);
  for (int i = threadIdx.x; i < kBins / 4; i += blockDim.x) {
    g1[i] = make_int4(i == kZeroBin / 4 ? zeros : 0, 0, 0, 0);
    g2[i] = make_int4(0, 0, 0, 0);
  }
  if (threadIdx.x == 0) {
    int32_t* cnt = zws + 2 * static_cast<int64_t>(rows) * kBins + 2 * row;
    cnt[0] = 0;
    cnt[1] = zeros;
  }
}

__global__ __launch_bounds__(kHistThreads) void pass1_hist_kernel(const float* __restrict__ score,
                                                                  int64_t score_stride, int width,
                                                                  const int16_t* __restrict__ mask,
                                                                  int64_t mask_stride,
                                                                  const int32_t* __restrict__ hist_lens,
                                                                  int32_t* __restrict__ zws, int rows) {
  __shared__ int sh[kBins];
  __shared__ int s_cnt[2];
  const int row = blockIdx.y;
  int h = hist_lens[row];
  h = h < width ? h : width;
  if (h <= kTopK) return;
  const int begin = blockIdx.x * kHistChunk;
  if (begin >= h) return;
  const int end = min(begin + kHistChunk, h);
  for (int i = threadIdx.x; i < kBins; i += kHistThreads) sh[i] = 0;
  if (threadIdx.x < 2) s_cnt[threadIdx.x] = 0;
  __syncthreads();
  const float* vals = score + static_cast<int64_t>(row) * score_stride;
  const int16_t* mrow = mask + static_cast<int64_t>(row) * mask_stride;
  int nz = 0, pos = 0;
  for (int i = begin + threadIdx.x; i < end; i += kHistThreads) {
    const bool set = (static_cast<uint16_t>(__ldg(mrow + (i >> 4))) >> (i & 15)) & 1u;
    if (set) {
      const uint32_t key = to_key(__ldg(vals + i));
      atomicAdd(&sh[key >> 20], 1);
      ++nz;
      pos += key > kZeroKey;
    }
  }
  nz = warp_sum(nz);
  pos = warp_sum(pos);
  if ((threadIdx.x & 31) == 0) {
    if (nz) atomicAdd(&s_cnt[0], nz);
    if (pos) atomicAdd(&s_cnt[1], pos);
  }
  __syncthreads();
  int32_t* g1 = zws + static_cast<int64_t>(row) * kBins;
  for (int i = threadIdx.x; i < kBins; i += kHistThreads)
    if (sh[i]) atomicAdd(&g1[i], sh[i]);
  if (threadIdx.x == 0) {
    int32_t* cnt = zws + 2 * static_cast<int64_t>(rows) * kBins + 2 * row;
    if (s_cnt[0]) {
      atomicSub(&g1[kZeroBin], s_cnt[0]);
      atomicSub(&cnt[1], s_cnt[0]);
    }
    if (s_cnt[1]) atomicAdd(&cnt[0], s_cnt[1]);
  }
}

bool use_vec(const float* score, int64_t width, int64_t stride) {
  return width % 4 == 0 && stride % 4 == 0 && reinterpret_cast<uintptr_t>(score) % 16 == 0;
}

int check_common(const float* score, int64_t rows, int64_t width, int64_t score_stride, const int16_t* mask,
                 int64_t mask_stride, const int32_t* lengths, const int32_t* pt, int64_t pt_stride, int64_t topk,
                 const int32_t* dst) {
  if (topk != kTopK) return HCU_ERR_ARG;
  if (rows < 0 || width < 0 || width > INT32_MAX / 2 || rows > INT32_MAX) return HCU_ERR_ARG;
  if (rows == 0) return HCU_OK;
  if (!score || !mask || !lengths || !pt || !dst) return HCU_ERR_ARG;
  if (score_stride < width || mask_stride < (width + 15) / 16 || pt_stride < 0) return HCU_ERR_ARG;
  return HCU_OK;
}

template <int kT, bool kVec>
void launch_split(const float* score, int rows, int width, int64_t score_stride, const int16_t* mask,
                  int64_t mask_stride, const int32_t* lengths, const int32_t* pt, int64_t pt_stride, int32_t* dst,
                  const int32_t* pre_ws, cudaStream_t stream, int splits);

template <int kT, bool kVec, bool kSorted>
void launch_rows_t(const float* score, int rows, int width, int64_t score_stride, const int16_t* mask,
                   int64_t mask_stride, const int32_t* lengths, const int32_t* pt, int64_t pt_stride, int32_t* dst,
                   uint32_t* dst_keys, const int32_t* pre_ws, cudaStream_t stream, int splits,
                   const int32_t* run_if = nullptr, int run_if_stride = 0) {
  const size_t smem = sizeof(TopkSmem<kT>);
  if (kSorted || splits <= 1) {
    // programmatic stream serialization: the grid may be scheduled while the previous kernel drains
    auto kern = topk_row_kernel<kT, kVec, kSorted, false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(rows));
    cfg.blockDim = dim3(kT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, score, score_stride, width, mask, mask_stride, lengths, pt, pt_stride, dst,
                       dst_keys, pre_ws, rows, 1, run_if, run_if_stride);
    return;
  }
  if constexpr (!kSorted) launch_split<kT, kVec>(score, rows, width, score_stride, mask, mask_stride, lengths, pt,
                                                 pt_stride, dst, pre_ws, stream, splits);
}

// One cluster of `splits` CTAs per row (splits <= kMaxClusterSplits).
template <int kT, bool kVec>
void launch_split(const float* score, int rows, int width, int64_t score_stride, const int16_t* mask,
                  int64_t mask_stride, const int32_t* lengths, const int32_t* pt, int64_t pt_stride, int32_t* dst,
                  const int32_t* pre_ws, cudaStream_t stream, int splits) {
  const size_t smem = sizeof(TopkSmem<kT>);
  uint32_t* dst_keys = nullptr;
  auto kern = topk_row_kernel<kT, kVec, false, true>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  // clusters of this size must fit the device (one query per size and device), else fewer CTAs per row
  static std::mutex mu;
  static std::vector<int> fits;  // [device * (kMaxClusterSplits + 1) + splits]: -1 unknown, 0 no, 1 yes
  int dev = 0;
  cudaGetDevice(&dev);
  for (; splits > 1; splits /= 2) {
    std::lock_guard<std::mutex> lk(mu);
    const size_t k = static_cast<size_t>(dev) * (kMaxClusterSplits + 1) + splits;
    if (fits.size() <= k) fits.resize(k + 1, -1);
    if (fits[k] < 0) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(static_cast<unsigned>(splits));
      q.blockDim = dim3(kT);
      q.dynamicSmemBytes = smem;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = static_cast<unsigned>(splits);
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.attrs = qa;
      q.numAttrs = 1;
      int n = 0;
      fits[k] = cudaOccupancyMaxActiveClusters(&n, kern, &q) == cudaSuccess && n > 0 ? 1 : 0;
      cudaGetLastError();  // a refused query is not a launch error
    }
    if (fits[k]) break;
  }
  if (splits <= 1) {
    launch_rows_t<kT, kVec, false>(score, rows, width, score_stride, mask, mask_stride, lengths, pt, pt_stride, dst,
                                   nullptr, pre_ws, stream, 1);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows * splits));
  cfg.blockDim = dim3(kT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, score, score_stride, width, mask, mask_stride, lengths, pt, pt_stride, dst, dst_keys,
                     pre_ws, rows, splits, static_cast<const int32_t*>(nullptr), 0);
}

template <int kT>
void launch_rows_sized(const float* score, int r, int w, int64_t score_stride, const int16_t* mask,
                       int64_t mask_stride, const int32_t* lengths, const int32_t* pt, int64_t pt_stride, int32_t* dst,
                       uint32_t* dst_keys, const int32_t* pre_ws, cudaStream_t stream, bool vec, bool sorted,
                       int splits, const int32_t* run_if, int run_if_stride) {
  if (vec && !sorted)
    launch_rows_t<kT, true, false>(score, r, w, score_stride, mask, mask_stride, lengths, pt, pt_stride, dst, dst_keys,
                                   pre_ws, stream, splits, run_if, run_if_stride);
  else if (vec)
    launch_rows_t<kT, true, true>(score, r, w, score_stride, mask, mask_stride, lengths, pt, pt_stride, dst, dst_keys,
                                  pre_ws, stream, splits, run_if, run_if_stride);
  else if (!sorted)
    launch_rows_t<kT, false, false>(score, r, w, score_stride, mask, mask_stride, lengths, pt, pt_stride, dst,
                                    dst_keys, pre_ws, stream, splits, run_if, run_if_stride);
  else
    launch_rows_t<kT, false, true>(score, r, w, score_stride, mask, mask_stride, lengths, pt, pt_stride, dst, dst_keys,
                                   pre_ws, stream, splits, run_if, run_if_stride);
}

int launch_rows(const float* score, int64_t rows, int64_t width, int64_t score_stride, const int16_t* mask,
                int64_t mask_stride, const int32_t* lengths, const int32_t* pt, int64_t pt_stride, int32_t* dst,
                uint32_t* dst_keys, const int32_t* pre_ws, cudaStream_t stream, bool sorted = false, int splits = 1,
                const int32_t* run_if = nullptr, int run_if_stride = 0) {
  const int w = static_cast<int>(width);
  const int r = static_cast<int>(rows);
  const bool vec = use_vec(score, width, score_stride);
  // narrow rows (or row parts), or rows up to 96K tokens when there are at least two per SM: 512
  // threads, two CTAs per SM (their latency-bound phases overlap; past 96K tokens the 4096-entry
  // candidate list of the 512-thread instance overflows too often)
  const int64_t part = (width + splits - 1) / splits;
  if (part <= kNarrowWidth || (rows >= 2 * static_cast<int64_t>(sm_count()) && part <= kManyRowsWidth))
    launch_rows_sized<512>(score, r, w, score_stride, mask, mask_stride, lengths, pt, pt_stride, dst, dst_keys, pre_ws,
                           stream, vec, sorted, splits, run_if, run_if_stride);
  else
    launch_rows_sized<1024>(score, r, w, score_stride, mask, mask_stride, lengths, pt, pt_stride, dst, dst_keys,
                            pre_ws, stream, vec, sorted, splits, run_if, run_if_stride);
  return launch_status();
}

// CTAs per row of the split entry points: the reference's heuristic
// (hcu_ops/__init__.py:52-57, sparse_mask_topk.cu:925-933) -- one per 8192 of
// width, no more than the SMs per row, at most max_splits -- capped at the
// portable cluster size.
int split_count(int64_t rows, int64_t width, int64_t max_splits) {
  int64_t s = std::max<int64_t>((width + 8191) / 8192, 1);
  s = std::min<int64_t>(s, sm_count() / std::max<int64_t>(rows, 1));
  s = std::min<int64_t>(s, std::min<int64_t>(max_splits, 64));
  s = std::min<int64_t>(s, kMaxClusterSplits);
  return static_cast<int>(std::max<int64_t>(s, 1));
}

// ---------------------------------------------------------------------------
// Context-parallel merge: P per-range top-2048 lists -> the global top-2048.
//
// Rank p of a KV-range split owns a contiguous global token range and emits
// (uint32 key, global index) for its local top-2048 in ascending token order
// (hcu_topk_keys), so the lists concatenated in rank order list every entry in
// ascending global index, and the global top-2048 under (key desc, index asc)
// is a subset of their union.  One 1024-thread CTA per row:
//   A  2048 strided samples of the concatenated lists give a lower bound lo of
//      the global threshold (the top-k kernel's sampled bound: a 12-bit and an
//      8-bit histogram, a sample rank 4 sigma + 4 below the expected one).
//   B  entries with key >= lo are appended in global index order to the
//      shared-memory candidate list (one block scan).
//   C  the top-k kernel's radix select and ordered write over the candidates
//      write the canonical order of the single-GPU top-k, so the CP result
//      equals the 1-GPU result exactly.
// Rows whose total visible length is at most 2048 keep every entry in index
// order (decided by the length, not the entry count: one range may hold all
// of a longer row's top-k).  A candidate list past kCandCap, or one shorter
// than 2048 (the bound missed), falls back to the digit descent over all entries.
// ---------------------------------------------------------------------------
constexpr int kMaxParts = 16;

// Entry c of a row's concatenated lists: part c >> lshift, position c & (2^lshift - 1);
// part p's list of row r starts at p * pstride + r * 2^lshift.
__device__ __forceinline__ int64_t merge_off(int c, int lshift, int64_t pstride, int row) {
  return static_cast<int64_t>(c >> lshift) * pstride + (static_cast<int64_t>(row) << lshift) +
         (c & ((1 << lshift) - 1));
}

// Valid entries (global index >= 0) of a row's concatenated lists: thread t
// owns entries [c0, c0 + per), in global index order across threads.
struct ListKeys {
  const uint32_t* keys;
  const int32_t* gidx;
  int c0, per, lshift, row;
  int64_t pstride;
  template <class F>
  __device__ __forceinline__ void operator()(F&& f) const {
    for (int i = 0; i < per; ++i) {
      const int64_t o = merge_off(c0 + i, lshift, pstride, row);
      if (__ldcg(gidx + o) >= 0) f(__ldcg(keys + o));
    }
  }
};

// Exact fallback of the merge (its candidate list overflowed or the sampled
// bound missed): the threshold by the digit descent over every valid entry,
// then, since each thread's entries are contiguous in index order, one block
// scan of (above, tie) counts places every selected entry.
template <int kT>
__device__ void merge_exact(TopkSmem<kT>& sm, const uint32_t* __restrict__ keys, const int32_t* __restrict__ gidx,
                            int per, int n_ent, int lshift, int64_t pstride, int row, int32_t* __restrict__ out,
                            int32_t* __restrict__ flag) {
  const int c0 = static_cast<int>(threadIdx.x) * per;
  per = max(0, min(per, n_ent - c0));
  const ListKeys src{keys, gidx, c0, per, lshift, row, pstride};
  int above = 0;
  const uint32_t thr = digit_descent(sm, src, kTopK, &above);
  const int remaining = kTopK - above;
  if (threadIdx.x == 0 && flag && sm.mark_any && sm.mark_max >= thr) atomicOr(flag, 1);  // a truncated list
  int na = 0, nt = 0;
  src([&](uint32_t k) {
    na += k > thr;
    nt += k == thr;
  });
  int total;
  const int ex = block_excl_scan<kT>(na | (nt << 16), sm.wtot, &total);
  int pa = ex & 0xFFFF, pq = ex >> 16;
  for (int i = 0; i < per; ++i) {
    const int64_t o = merge_off(c0 + i, lshift, pstride, row);
    const int g = __ldcg(gidx + o);
    if (g < 0) continue;
    const uint32_t k = __ldcg(keys + o);
    if (k > thr) {
      out[pa++] = g;
    } else if (k == thr) {
      if (pq < remaining) out[above + pq] = g;
      ++pq;
    }
  }
}

// Lists of 2^lshift entries per (part, row), part p at p * pstride; flag
// (optional): set when a row longer than kTopK holds fewer than kTopK entries
// (a caller-side bound missed), instead of the sticky bad-input status, or
// when the row's threshold is not above the key of a truncation marker (entry
// -2: the largest key its list may have dropped);
// short_identity: rows of at most kTopK visible tokens [0, len) output
// 0, 1, .., len - 1 without reading the lists (identity page table).
// The merge of one row (every thread of the CTA calls it), result into out[0, kTopK).
template <int kT>
__device__ __noinline__ void merge_row(TopkSmem<kT>& sm, const uint32_t* __restrict__ keys,
                                       const int32_t* __restrict__ gidx, int parts, int lshift, int64_t pstride,
                                       const int32_t* __restrict__ lengths, int row, int32_t* __restrict__ out,
                                       int32_t* __restrict__ flag, int short_identity) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int w = tid >> 5;
  if (short_identity) {
    const int vl = __ldg(lengths + row);
    if (vl <= kTopK) {
      for (int i = tid; i < kTopK; i += kT) out[i] = i < vl ? i : -1;
      return;
    }
  }
  for (int i = tid; i < 2 * 512; i += kT) (&sm.hb[0][0])[i] = 0;
  if (tid == 0) {
    sm.mark_any = 0;
    sm.mark_max = 0u;
  }

  const int n_ent = parts << lshift;  // entries of the row's concatenated lists
  // ---- A: lower bound lo from 2048 evenly spaced samples of the concatenated lists ----
  for (int i = tid; i < kBins; i += kT) sm.hist[i] = 0;
  __syncthreads();
  constexpr int kMs = 2048;  // samples
  uint32_t sk[kMs / kT];
#pragma unroll
  for (int j = 0; j < kMs / kT; ++j) {
    const int c = static_cast<int>(static_cast<int64_t>(tid + j * kT) * n_ent / kMs) + n_ent / (2 * kMs);
    const int64_t o = merge_off(min(c, n_ent - 1), lshift, pstride, row);
    sk[j] = __ldcg(gidx + o) >= 0 ? __ldcg(keys + o) : 0u;  // a missing entry ranks below every key
    atomicAdd(&sm.hist[sk[j] >> 20], 1);
  }
  __syncthreads();
  // sample rank (1 = largest) 4 sigma + 4 below the threshold's expected sample rank
  const float t = static_cast<float>(kMs) * static_cast<float>(kTopK) / static_cast<float>(n_ent);
  const int r_lo = min(kMs, static_cast<int>(ceilf(t + 4.f * sqrtf(t) + 4.f)));
  block_rank_bin<kT, kBins>(sm.hist, r_lo, sm.wtot, sm.res);
  const uint32_t b1 = static_cast<uint32_t>(sm.res[0]);
  const int need = r_lo - sm.res[1];
#pragma unroll
  for (int j = 0; j < kMs / kT; ++j)
    if ((sk[j] >> 20) == b1) atomicAdd(&sm.hb[0][(sk[j] >> 12) & 0xFFu], 1);
  __syncthreads();
  if (w == 0) warp_find<256>(sm.hb[0], need, sm.res);
  __syncthreads();
  uint32_t lo = (b1 << 20) | (static_cast<uint32_t>(sm.res[0]) << 12);
  if (tid < 256) sm.hb[0][tid] = 0;  // ordered before the select by the barriers below
  const bool short_row = __ldg(lengths + row) <= kTopK;
  if (short_row) lo = 0u;  // keep every entry

  // ---- B: entries with key >= lo, appended in global index order ----
  const int per = (n_ent + kT - 1) / kT;  // <= 32
  const int c0 = tid * per;
  // thread t: entries [t * per, (t + 1) * per), per <= 32; loads go out 8 at a time
  int na = 0, nv = 0, mk = 0;
  uint32_t kmax = 0u, cbits = 0u, mmax = 0u;
  for (int i0 = 0; i0 < per; i0 += 8) {
    uint32_t kk[8];
    int gg[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      gg[u] = -1;
      kk[u] = 0u;
      if (i0 + u < per && c0 + i0 + u < n_ent) {
        const int64_t o = merge_off(c0 + i0 + u, lshift, pstride, row);
        kk[u] = __ldcg(keys + o);
        gg[u] = __ldcg(gidx + o);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (gg[u] >= 0) {
        ++nv;
        if (kk[u] >= lo) {
          ++na;
          cbits |= 1u << (i0 + u);
          kmax = kk[u] > kmax ? kk[u] : kmax;
        }
      } else if (gg[u] == -2) {  // marker of a truncated list: the largest key it may have dropped
        mk = 1;
        mmax = kk[u] > mmax ? kk[u] : mmax;
      }
    }
  }
  int packed_total;
  const int packed = block_excl_scan<kT>(na | (nv << 16), sm.wtot, &packed_total);
  const int n = packed_total & 0xFFFF;
  const int total = static_cast<int>(static_cast<uint32_t>(packed_total) >> 16);
  int pos = packed & 0xFFFF;
  if (n <= Tk<kT>::kCandCap) {
    for (int i0 = 0; i0 < per && (cbits >> i0); i0 += 8) {
      uint32_t kk[8];
      int gg[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if ((cbits >> (i0 + u)) & 1u) {
          const int64_t o = merge_off(c0 + i0 + u, lshift, pstride, row);
          kk[u] = __ldcg(keys + o);
          gg[u] = __ldcg(gidx + o);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if ((cbits >> (i0 + u)) & 1u) {
          sm.cand_key[pos] = kk[u];
          sm.cand_pid[pos] = gg[u];
          ++pos;
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t y = __shfl_xor_sync(0xffffffffu, kmax, o);
    kmax = y > kmax ? y : kmax;
    const uint32_t z = __shfl_xor_sync(0xffffffffu, mmax, o);
    mmax = z > mmax ? z : mmax;
  }
  if (lane == 0) sm.wmax[w] = kmax;
  if (__any_sync(0xffffffffu, mk) && lane == 0) {
    atomicOr(&sm.mark_any, 1);
    atomicMax(&sm.mark_max, mmax);
  }
  __syncthreads();

  if (short_row || total < kTopK) {
    // all entries in index order; fewer than 2048 entries for a longer row is inconsistent input,
    // or (with flag) a caller's bound that missed
    if (!short_row && tid == 0) {
      if (flag)
        atomicOr(flag, 1);
      else
        atomicOr(&g_hcu_status, HCU_STATUS_BAD_INPUT);
    }
    for (int i = tid; i < kTopK; i += kT) out[i] = i < n && i < Tk<kT>::kCandCap ? sm.cand_pid[i] : -1;
    return;
  }
  if (n > Tk<kT>::kCandCap || n < kTopK) {  // list overflow, or the sampled bound missed
    merge_exact(sm, keys, gidx, per, n_ent, lshift, pstride, row, out, flag);
    return;
  }
  // ---- C: select and ordered write over the candidates ----
  int above = 0;
  const uint32_t thr = select_candidates(sm, n, lo, &above);
  if (tid == 0 && flag && sm.mark_any && sm.mark_max >= thr) atomicOr(flag, 1);  // a truncated list
  write_candidates<kT, false>(sm, n, thr, above, out, nullptr);
}

template <int kT>
__global__ __launch_bounds__(kT, 1024 / kT) void cp_merge_kernel(const uint32_t* __restrict__ keys,
                                                                const int32_t* __restrict__ gidx, int parts,
                                                                int lshift, int64_t pstride,
                                                                const int32_t* __restrict__ lengths,
                                                                int32_t* __restrict__ dst, int32_t* __restrict__ flag,
                                                                int short_identity) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TopkSmem<kT>& sm = *reinterpret_cast<TopkSmem<kT>*>(smem_raw);
  const int row = blockIdx.x;
  merge_row(sm, keys, gidx, parts, lshift, pstride, lengths, row, dst + static_cast<int64_t>(row) * kTopK, flag,
            short_identity);
}
// ---------------------------------------------------------------------------
// Context-parallel candidate filter (the bounded exchange of hcu_ops/cp.py).
//
// Instead of a local top-2048 per range, each rank keeps only the tokens that
// can still be in the row's global top-2048: those with key >= b, where b is
// the minimum over ranks of a sampled estimate of the row's global threshold
// on each rank's own range (cp_bound_kernel, then an all-reduce MIN).  The
// filter (cp_filter_kernel) emits every such token in token order into a short
// fixed-capacity list.  The union is exact iff it holds at least kTopK entries
// per row (then the global threshold is >= b, so every token of the global
// top-k passed the filter) and no list overflowed; the merge and the filter
// flag the rows where either fails, and the caller then runs the exact path.
// ---------------------------------------------------------------------------
constexpr int kBoundWarps = 8;        // rows per CTA of the bound kernel (one warp each)
constexpr int kBoundSamples = 1024;   // samples of a row's local range

struct __align__(16) BoundSmem {
  uint32_t k[kBoundWarps][kBoundSamples];
  alignas(16) int h[kBoundWarps][256];
  int res[kBoundWarps][4];
};

// Bound of row `row` on this range, as an order-preserving int32 (key ^ 0x80000000):
// the sample key of rank r_lo = t + 3 sqrt(t) + 2 (1 = largest) among m
// samples of the local range (m / 4 evenly spaced groups of 4 consecutive
// tokens, one 16-byte load and one mask word each; every token when n <= m),
// t = kTopK * m / total the expected sample rank of the global threshold.  The largest key (no constraint on the minimum)
// for rows of at most kTopK visible tokens (the merge writes them as the
// identity), for empty ranges, and for ranges expected to hold less than one
// token of the row's top-kTopK (kTopK * n < total): their few tokens are
// covered by the other ranges' margins, and their noisy estimate would pull
// every range's bound down.  Exactness never rests on the estimate: the merge
// checks that the union holds kTopK entries.
template <bool kVec>
__device__ __forceinline__ uint32_t row_bound(BoundSmem& sm, const float* __restrict__ score, int64_t score_stride,
                                              int width, const int16_t* __restrict__ mask, int64_t mask_stride,
                                              const int32_t* __restrict__ lengths,
                                              const int32_t* __restrict__ totals, int row) {
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  int n = __ldg(lengths + row);
  n = n < 0 ? 0 : (n > width ? width : n);
  const int total = __ldg(totals + row);
  uint32_t v = 0xFFFFFFFFu;
  if (total > kTopK && static_cast<int64_t>(kTopK) * n >= total) {
    v = 0u;
    const int m = n <= kBoundSamples ? n : kBoundSamples;
    const float t = static_cast<float>(kTopK) * static_cast<float>(m) / static_cast<float>(total);
    const int r_lo = static_cast<int>(ceilf(t + 3.f * sqrtf(t) + 2.f));
    if (r_lo < m) {
      const float* vals = score + static_cast<int64_t>(row) * score_stride;
      const int16_t* mrow = mask + static_cast<int64_t>(row) * mask_stride;
      uint32_t* ks = sm.k[w];
      if (n <= kBoundSamples) {  // every token
        for (int i = lane; i < n; i += 32) {
          const bool set = (static_cast<uint16_t>(__ldg(mrow + (i >> 4))) >> (i & 15)) & 1u;
          ks[i] = set ? to_key(__ldg(vals + i)) : kZeroKey;
        }
      } else {  // group g: tokens i .. i + 3 < n, i = ((2g + 1) n / (2 m / 4)) rounded down to a multiple of 4
        constexpr int kGroups = kBoundSamples / 4;
        for (int g = lane; g < kGroups; g += 32) {
          const int i = min(static_cast<int>((2 * static_cast<int64_t>(g) + 1) * n / (2 * kGroups)), n - 4) & ~3;
          const uint32_t mb = static_cast<uint16_t>(__ldg(mrow + (i >> 4))) >> (i & 15);
          float f[4];
          if constexpr (kVec) {
            const float4 q = __ldg(reinterpret_cast<const float4*>(vals + i));
            f[0] = q.x; f[1] = q.y; f[2] = q.z; f[3] = q.w;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) f[e] = __ldg(vals + i + e);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) ks[4 * g + e] = ((mb >> e) & 1u) ? to_key(f[e]) : kZeroKey;
        }
      }
      // r_lo-th largest sample key: four 8-bit radix passes over the warp's samples
      uint32_t pre = 0u;
      int need = r_lo;
      int* h = sm.h[w];
      for (int pass = 0; pass < 4; ++pass) {
        const int sh = 24 - 8 * pass;
        for (int i = lane; i < 256; i += 32) h[i] = 0;
        __syncwarp();
        for (int j = lane; j < m; j += 32) {
          const uint32_t k = ks[j];
          if (pass == 0 || (k >> (sh + 8)) == pre) atomicAdd(&h[(k >> sh) & 0xFFu], 1);
        }
        __syncwarp();
        warp_find<256>(h, need, sm.res[w]);
        __syncwarp();
        pre = (pre << 8) | static_cast<uint32_t>(sm.res[w][0]);
        need -= sm.res[w][1];
        __syncwarp();
      }
      v = pre;
    }
  }
  return v;
}

template <bool kVec>
__global__ __launch_bounds__(kBoundWarps * 32) void cp_bound_kernel(
    const float* __restrict__ score, int64_t score_stride, int width, const int16_t* __restrict__ mask,
    int64_t mask_stride, const int32_t* __restrict__ lengths, const int32_t* __restrict__ totals, int rows,
    int32_t* __restrict__ bounds) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BoundSmem& sm = *reinterpret_cast<BoundSmem*>(smem_raw);
  const int row = blockIdx.x * kBoundWarps + (threadIdx.x >> 5);
  if (row >= rows) return;  // whole warps; the kernel has no block barrier
  const uint32_t v = row_bound<kVec>(sm, score, score_stride, width, mask, mask_stride, lengths, totals, row);
  if ((threadIdx.x & 31) == 0) bounds[row] = static_cast<int32_t>(v ^ kZeroKey);
}

// One CTA per row: every token of [0, len) with key >= the row's bound, in
// token order, as (key, page-table entry) into list slots [0, cap) of the row
// (key 0 / entry -1 pads); row r's list starts at (r / rows_per_block) *
// block_stride + (r % rows_per_block) * cap (so a row-sharded exchange buffer
// is written in place); counts[row] (optional) = all such tokens.  More than
// cap of them: with cap = kTopK the list holds the range's top-kTopK among them
// (exact for the merge); with cap < kTopK its top-(cap - 1) and a marker slot
// (entry -2, key = the largest key it may have dropped) that the merge checks;
// past the candidate capacity *flag |= 1.
template <int kT, bool kVec>
__device__ __noinline__ int filter_row(TopkSmem<kT>& sm, const float* __restrict__ vals,
                                       const int16_t* __restrict__ mrow, const int32_t* __restrict__ src, int len,
                                       uint32_t lo, int cap, uint32_t* __restrict__ ok, int32_t* __restrict__ og,
                                       int32_t* __restrict__ flag) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int w = tid >> 5;
  uint32_t b0[16], valid0 = 0u;
  const uint32_t mw0 = load16_raw<kVec>(vals, mrow, w * (32 * kLaneTok) + lane * kLaneTok, len, b0, valid0);
  for (int i = tid; i < 2 * 512; i += kT) (&sm.hb[0][0])[i] = 0;  // the select's digit histograms
  const int n = lo > kZeroKey ? collect_candidates<kT, kVec, true>(vals, mrow, src, 0, len, lo, sm, b0, mw0, valid0)
                              : collect_candidates<kT, kVec, false>(vals, mrow, src, 0, len, lo, sm, b0, mw0, valid0);
  cp_async_wait_all();
  __syncthreads();
  if (n > cap && n <= Tk<kT>::kCandCap) {
    // More candidates than slots.  cap = kTopK: the range's exact top-kTopK among them, in token
    // order, holds every token of the row's global top-kTopK that lies in this range.  cap < kTopK:
    // its top-(cap - 1) in token order and, in the last slot, a marker (entry -2) whose key is the
    // (cap - 1)-th largest key: every dropped token has a key <= it, and the merge accepts the
    // row only when the global threshold is above every marker.
    const int k = cap == kTopK ? kTopK : cap - 1;
    int above = 0;
    const uint32_t thr = select_candidates(sm, n, lo, &above, k);
    write_candidates<kT, true>(sm, n, thr, above, og, ok, k);
    if (k < cap && tid == 0) {
      ok[cap - 1] = thr;
      og[cap - 1] = -2;
    }
  } else {
    const int kept = min(n, cap);  // cap <= kTopK <= kCandCap: every kept entry is in the list
    for (int i = tid; i < cap; i += kT) {
      ok[i] = i < kept ? sm.cand_key[i] : 0u;
      og[i] = i < kept ? sm.cand_pid[i] : -1;
    }
    if (tid == 0 && n > cap) atomicOr(flag, 1);  // past the candidate capacity
  }
  return n;
}

// One row of the filter on one warp: the tokens of [0, len) with key >= lo, in token order, as (key,
// page-table entry) into slots [0, cap) with key 0 / entry -1 pads -- the list filter_row writes
// when it holds at most cap entries.  Lanes take 16 consecutive tokens, two chunks in flight; for a
// positive lo the test is one signed compare of the raw bits.  `stage`: this warp's 32 x 16 words of
// shared memory.  Returns the count (uniform); above cap nothing is padded and the caller runs
// filter_row on the row instead (the list then takes the range's top entries and a marker).
template <bool kVec>
__device__ __forceinline__ int filter_row_warp(const float* __restrict__ vals, const int16_t* __restrict__ mrow,
                                               const int32_t* __restrict__ src, int len, uint32_t lo, int cap,
                                               uint32_t* __restrict__ ok, int32_t* __restrict__ og,
                                               uint32_t* stage) {
  const int lane = threadIdx.x & 31;
  const bool pos = lo > kZeroKey;
  const int lo_bits = static_cast<int>(lo & 0x7FFFFFFFu);
  int n = 0;  // uniform over the warp
  for (int c0 = 0; c0 < len; c0 += 2 * 32 * kLaneTok) {
    uint32_t b[2][16], valid[2], mw[2];
#pragma unroll
    for (int u = 0; u < 2; ++u)
      mw[u] = load16_raw<kVec>(vals, mrow, c0 + (u * 32 + lane) * kLaneTok, len, b[u], valid[u]);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i0 = c0 + (u * 32 + lane) * kLaneTok;
      uint32_t hit = 0u;
      if (pos) {
#pragma unroll
        for (int e = 0; e < 16; ++e) hit |= (static_cast<int>(b[u][e]) >= lo_bits ? 1u : 0u) << e;
        hit &= mw[u] & valid[u];
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint32_t k = ((mw[u] >> e) & 1u) ? key_of(__uint_as_float(b[u][e])) : kZeroKey;
          b[u][e] = k;
          hit |= (((valid[u] >> e) & 1u) && k >= lo) ? (1u << e) : 0u;
        }
      }
      const int c = __popc(hit);
      const int inc = warp_incl_scan(c);
      int at = n + inc - c;
      n += __shfl_sync(0xffffffffu, inc, 31);
      if (hit && at < cap) {  // the lane's words through shared memory, read back at the set bits
        uint4* st4 = reinterpret_cast<uint4*>(stage + lane * kLaneTok);
#pragma unroll
        for (int q = 0; q < 4; ++q) st4[q] = make_uint4(b[u][4 * q], b[u][4 * q + 1], b[u][4 * q + 2], b[u][4 * q + 3]);
        const uint32_t* sw = stage + lane * kLaneTok;
        const uint32_t kbit = pos ? kZeroKey : 0u;
        do {
          const int e = __ffs(hit) - 1;
          hit &= hit - 1u;
          if (at < cap) {
            ok[at] = sw[e] | kbit;
            og[at] = __ldg(src + i0 + e);
          }
          ++at;
        } while (hit);
      }
    }
  }
  if (n <= cap)
    for (int i = n + lane; i < cap; i += 32) {
      ok[i] = 0u;
      og[i] = -1;
    }
  return n;
}

// Rows of a CTA per warp pass: at most this many (a bitmap of the rows whose list overflowed).
constexpr int kFilterRowsPerCta = 4096;

template <int kT, bool kVec>
__global__ __launch_bounds__(kT, 1024 / kT) void cp_filter_kernel(
    const float* __restrict__ score, int64_t score_stride, int width, const int16_t* __restrict__ mask,
    int64_t mask_stride, const int32_t* __restrict__ lengths, const int32_t* __restrict__ pt, int64_t pt_stride,
    const int32_t* __restrict__ bounds, int cap, uint32_t* __restrict__ out_keys, int32_t* __restrict__ out_gidx,
    int rows_per_block, int64_t block_stride, int32_t* __restrict__ counts, int32_t* __restrict__ flag, int rows,
    int warp_pass) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TopkSmem<kT>& sm = *reinterpret_cast<TopkSmem<kT>*>(smem_raw);
  __shared__ uint32_t ovf[kFilterRowsPerCta / 32];  // rows (by their index in this CTA) left to filter_row
  auto lo_of = [&](int row) { return static_cast<uint32_t>(__ldg(bounds + row)) ^ kZeroKey; };
  auto off_of = [&](int row) {
    return (row / rows_per_block) * block_stride + static_cast<int64_t>(row % rows_per_block) * cap;
  };
  auto len_of = [&](int row) {
    const int len = __ldg(lengths + row);
    return len < 0 ? 0 : (len > width ? width : len);
  };
  // persistent CTAs, rows strided over the grid; with warp_pass, first a warp per row
  const int nk = (rows - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  if (warp_pass) {
    for (int i = threadIdx.x; i < kFilterRowsPerCta / 32; i += kT) ovf[i] = 0u;
    __syncthreads();
    const int w = threadIdx.x >> 5;
    uint32_t* stage = reinterpret_cast<uint32_t*>(&sm.scr[0][0]) + w * 32 * kLaneTok;
    for (int k = w; k < nk; k += kT / 32) {
      const int row = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
      const int64_t off = off_of(row);
      const int n = filter_row_warp<kVec>(score + static_cast<int64_t>(row) * score_stride,
                                          mask + static_cast<int64_t>(row) * mask_stride,
                                          pt + static_cast<int64_t>(row) * pt_stride, len_of(row), lo_of(row), cap,
                                          out_keys + off, out_gidx + off, stage);
      if ((threadIdx.x & 31) == 0) {
        if (n > cap)
          atomicOr(&ovf[k >> 5], 1u << (k & 31));
        else if (counts)
          counts[row] = n;
      }
    }
    __syncthreads();
  }
  for (int k = 0; k < nk; ++k) {
    if (warp_pass && !((ovf[k >> 5] >> (k & 31)) & 1u)) continue;  // uniform: shared state
    const int row = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
    const int64_t off = off_of(row);
    const int n = filter_row<kT, kVec>(sm, score + static_cast<int64_t>(row) * score_stride,
                                       mask + static_cast<int64_t>(row) * mask_stride,
                                       pt + static_cast<int64_t>(row) * pt_stride, len_of(row), lo_of(row), cap,
                                       out_keys + off, out_gidx + off, flag);
    if (threadIdx.x == 0 && counts) counts[row] = n;
    __syncthreads();  // the row's shared state is read out before the next row reuses it
  }
}

// ---------------------------------------------------------------------------
// Fused prefill top-k, last step: the ragged logits kernel appended every
// visible token at or above the row's bound to the row's list (unordered
// (key, token) pairs, cnt[row] of them).  One CTA per row selects the top
// kTopK of the list (the radix select over u = key - lo) and writes them in
// the canonical order -- tokens above the threshold in ascending token order,
// then threshold ties in ascending token order -- through token bitmaps in
// shared memory.  The result equals the top-k of the materialised logits iff
// the list is complete (cnt <= cap) and holds at least kTopK tokens; other
// rows raise *flag (the caller's exact path then rewrites every row).  Rows of
// at most kTopK visible tokens are written as the identity.  256-thread CTAs
// with the list's keys in shared memory: several rows per SM hide the per-row
// latency of the load, the radix rounds and the ordered write.
// ---------------------------------------------------------------------------
constexpr int kFusedMaxWidth = 131072;  // two token bitmaps of the row in shared memory
constexpr int kFusedCap = 8192;         // candidate list capacity of the select

// Fused prefill bound: one warp per row over every sampled score of the row
// (its n = e_s[row] sampled tokens, at most kFusedSamples), the sample key of
// rank t + 5 sqrt(t) + 5 with t = kTopK * n / len the expected sample rank of
// the row's threshold (the wide margin keeps the chance that a row's list
// misses the threshold, which sends the whole call down the exact path, far
// below one in the thousands of rows of a prefill chunk).  Rows of at most
// kTopK tokens and rows whose sample cannot bound anything give the largest
// key.  Output: order-preserving int32 (key ^ 0x80000000).
constexpr int kFusedSamples = 4096;  // 131072 tokens / 32
constexpr int kFusedBoundWarps = 4;

struct __align__(16) FusedBoundSmem {
  uint32_t k[kFusedBoundWarps][kFusedSamples];
  alignas(16) int h[kFusedBoundWarps][256];
  int res[kFusedBoundWarps][4];
};

__global__ __launch_bounds__(kFusedBoundWarps * 32) void fused_bound_kernel(
    const float* __restrict__ score, int64_t score_stride, const int16_t* __restrict__ mask, int64_t mask_stride,
    const int32_t* __restrict__ e_s, const int32_t* __restrict__ row_end, int width, int rows,
    int32_t* __restrict__ bounds) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FusedBoundSmem& sm = *reinterpret_cast<FusedBoundSmem*>(smem_raw);
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int row = blockIdx.x * kFusedBoundWarps + w;
  if (row >= rows) return;  // whole warps; no block barrier below
  int len = __ldg(row_end + row);
  len = len < 0 ? 0 : (len > width ? width : len);
  const int n = min(__ldg(e_s + row), kFusedSamples);
  uint32_t v = 0xFFFFFFFFu;
  if (len > kTopK && n > 0) {
    const float t = static_cast<float>(kTopK) * static_cast<float>(n) / static_cast<float>(len);
    const int r_lo = static_cast<int>(ceilf(t + 5.f * sqrtf(t) + 5.f));
    if (r_lo <= n) {
      const float* vals = score + static_cast<int64_t>(row) * score_stride;
      const int16_t* mrow = mask + static_cast<int64_t>(row) * mask_stride;
      uint32_t* ks = sm.k[w];
      for (int i = lane; i < n; i += 32) {
        const bool set = (static_cast<uint16_t>(__ldg(mrow + (i >> 4))) >> (i & 15)) & 1u;
        ks[i] = set ? to_key(__ldg(vals + i)) : kZeroKey;
      }
      uint32_t pre = 0u;
      int need = r_lo;
      int* h = sm.h[w];
      for (int pass = 0; pass < 4; ++pass) {  // the r_lo-th largest key, 8 bits at a time
        const int sh = 24 - 8 * pass;
        for (int i = lane; i < 256; i += 32) h[i] = 0;
        __syncwarp();
        for (int j = lane; j < n; j += 32) {
          const uint32_t k = ks[j];
          if (pass == 0 || (k >> (sh + 8)) == pre) atomicAdd(&h[(k >> sh) & 0xFFu], 1);
        }
        __syncwarp();
        warp_find<256>(h, need, sm.res[w]);
        __syncwarp();
        pre = (pre << 8) | static_cast<uint32_t>(sm.res[w][0]);
        need -= sm.res[w][1];
        __syncwarp();
      }
      v = pre;
    }
  }
  if (lane == 0) bounds[row] = static_cast<int32_t>(v ^ kZeroKey);
}

// Keys only (the tokens are re-read from the list, L2-resident, once the threshold is known), and
// the two token bitmaps sized to the row width after the struct, so that four 256-thread CTAs fit
// an SM at the benchmark widths.
template <int kT>
struct __align__(16) FusedSelSmem {
  uint32_t cand_key[kFusedCap];
  alignas(16) int hb[2][512];
  uint32_t wmax[kT / 32];
  int wtot[32];
  int res[4];
  alignas(16) uint32_t bm[1];  // 2 x ceil(width / 32) words: tokens above the threshold, then threshold ties
};

template <int kT>
__global__ __launch_bounds__(kT, 1024 / kT) void fused_select_kernel(
    const int2* __restrict__ cand, const int32_t* __restrict__ cnt, int cap, const int32_t* __restrict__ row_end,
    int width, const int32_t* __restrict__ bounds, int all_len, const int32_t* __restrict__ pt, int64_t pt_stride,
    int32_t* __restrict__ dst, int32_t* __restrict__ flag, int flag_per_row) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FusedSelSmem<kT>& sm = *reinterpret_cast<FusedSelSmem<kT>*>(smem_raw);
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int w = tid >> 5;
  int len = __ldg(row_end + row);
  len = len < 0 ? 0 : (len > width ? width : len);
  const int32_t* src = pt + static_cast<int64_t>(row) * pt_stride;
  int32_t* out = dst + static_cast<int64_t>(row) * kTopK;
  // flag_per_row: every row's word of flag is written (1: the row is left to the exact path), else
  // one word for the call, raised by any failing row
  if (len <= kTopK) {
    for (int i = tid; i < kTopK; i += kT) out[i] = i < len ? src[i] : -1;
    if (flag_per_row && tid == 0) flag[row] = 0;
    return;
  }
  const int n = __ldcg(cnt + row);
  if (n > cap || n < kTopK || n > kFusedCap) {  // incomplete list or a bound above the threshold
    if (tid == 0) {
      if (flag_per_row)
        flag[row] = 1;
      else
        atomicOr(flag, 1);
    }
    return;
  }
  if (flag_per_row && tid == 0) flag[row] = 0;
  const uint32_t lo = len <= all_len ? 0u : static_cast<uint32_t>(__ldg(bounds + row)) ^ kZeroKey;
  const int nw = (len + 31) >> 5;
  uint32_t* abm = sm.bm;       // tokens above the threshold
  uint32_t* tbm = sm.bm + nw;  // threshold ties
  for (int i = tid; i < 2 * nw; i += kT) abm[i] = 0u;
  for (int i = tid; i < 2 * 512; i += kT) (&sm.hb[0][0])[i] = 0;
  const int2* lst = cand + static_cast<int64_t>(row) * cap;
  uint32_t m = 0u;
  for (int i = tid; i < n; i += kT) {
    const uint32_t k = static_cast<uint32_t>(__ldcg(&lst[i].x));
    sm.cand_key[i] = k;
    m = k > m ? k : m;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t y = __shfl_xor_sync(0xffffffffu, m, o);
    m = y > m ? y : m;
  }
  if (lane == 0) sm.wmax[w] = m;
  __syncthreads();
  int above = 0;
  const uint32_t thr = select_candidates_in<kT>(sm, n, lo, &above);
  for (int i = tid; i < n; i += kT) {
    const uint32_t k = sm.cand_key[i];
    if (k < thr) continue;
    const int t = __ldcg(&lst[i].y);
    if (k > thr)
      atomicOr(abm + (t >> 5), 1u << (t & 31));
    else if (k == thr)
      atomicOr(tbm + (t >> 5), 1u << (t & 31));
  }
  __syncthreads();
  // thread tid takes words [i0, i1) of both bitmaps: its above tokens go after the above tokens of
  // lower words, its ties after the lower words' ties (the first kTopK - above ties are kept)
  const int per = (nw + kT - 1) / kT;
  const int i0 = min(nw, tid * per);
  const int i1 = min(nw, i0 + per);
  int na = 0, nt = 0;
  for (int i = i0; i < i1; ++i) {
    na += __popc(abm[i]);
    nt += __popc(tbm[i]);
  }
  int total;
  const int ex = block_excl_scan<kT>(na | (nt << 16), sm.wtot, &total);
  int ea = ex & 0xFFFF;
  int et = ex >> 16;
  const int remaining = kTopK - above;
  // the output's tokens in the canonical order into the key array (the keys are no longer read),
  // then every page-table entry at once (kTopK / kT independent loads a thread, not a chain)
  int* const otok = reinterpret_cast<int*>(sm.cand_key);
  for (int i = i0; i < i1; ++i) {
    uint32_t a = abm[i];
    while (a) {
      const int b = __ffs(a) - 1;
      a &= a - 1u;
      otok[ea++] = (i << 5) + b;
    }
    uint32_t t = tbm[i];
    while (t && et < remaining) {
      const int b = __ffs(t) - 1;
      t &= t - 1u;
      otok[above + et++] = (i << 5) + b;
    }
  }
  __syncthreads();
  int32_t v[kTopK / kT];
#pragma unroll
  for (int q = 0; q < kTopK / kT; ++q) v[q] = __ldg(src + otok[tid + q * kT]);
#pragma unroll
  for (int q = 0; q < kTopK / kT; ++q) out[tid + q * kT] = v[q];
}

// ---------------------------------------------------------------------------
// List top-k for many rows (at least two rows per SM: prefill chunks, the
// one-GPU context-parallel case).  The block-per-row kernel keeps two rows in
// flight per SM and its per-row latency bounds it; here the row stream is
// split from the select:
//   1. list_bound_kernel, one warp per row: kListSamples samples of the row
//      (evenly spaced groups of 4 consecutive tokens) and the sample key of
//      rank t + 5 sqrt(t) + 5, t = kTopK * kListSamples / len the expected
//      sample rank of the row's threshold, as the row's bound lo;
//   2. list_collect_kernel, one warp per row: streams the row and appends
//      every visible token with key >= lo, as (key, token), to the row's list
//      (rows of at most all_len tokens list every token);
//   3. fused_select_kernel: the top kTopK of each list in the canonical order,
//      with a word per row telling whether the list proved exactness;
//   4. the block-per-row kernel, predicated per row on those words, rewrites
//      the rows whose list missed or overflowed.
// The stream runs with tens of rows in flight per SM, so the pass reads the
// scores at close to the HBM rate; the select reads only the short lists.
// ---------------------------------------------------------------------------
constexpr int kListSamples = 2048;
constexpr int kListBoundWarps = 8;
constexpr int kListAllLen = 4096;  // rows of at most this many tokens list every token

struct __align__(16) ListBoundSmem {
  uint32_t k[kListBoundWarps][kListSamples];
  alignas(16) int h[kListBoundWarps][256];
  int res[kListBoundWarps][4];
};

template <bool kVec>
__global__ __launch_bounds__(kListBoundWarps * 32) void list_bound_kernel(
    const float* __restrict__ score, int64_t score_stride, int width, const int16_t* __restrict__ mask,
    int64_t mask_stride, const int32_t* __restrict__ lengths, int rows, int32_t* __restrict__ bounds) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ListBoundSmem& sm = *reinterpret_cast<ListBoundSmem*>(smem_raw);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int row = blockIdx.x * kListBoundWarps + w;
  if (row >= rows) return;  // whole warps; no block barrier below
  int len = __ldg(lengths + row);
  len = len < 0 ? 0 : (len > width ? width : len);
  uint32_t v = 0u;  // rows listed whole ignore it
  if (len > kListAllLen) {
    const float t = static_cast<float>(kTopK) * static_cast<float>(kListSamples) / static_cast<float>(len);
    const int r_lo = static_cast<int>(ceilf(t + 5.f * sqrtf(t) + 5.f));  // < kListSamples for len > kListAllLen
    const float* vals = score + static_cast<int64_t>(row) * score_stride;
    const int16_t* mrow = mask + static_cast<int64_t>(row) * mask_stride;
    uint32_t* ks = sm.k[w];
    // kListSamples / 32 evenly spaced blocks of 32 consecutive tokens (one 128-byte line each, so
    // the sample reads stay a small share of the row's bytes); 8 lanes per block, 4 tokens a lane
    constexpr int kGroups = kListSamples / 4;
    constexpr int kBlocks = kListSamples / 32;
    const float stride_b = static_cast<float>(len) / static_cast<float>(kBlocks);
    const int blast = (len - 32) & ~31;
    uint32_t kmax = 0u, kmin = 0xFFFFFFFFu;
#pragma unroll 4
    for (int g = lane; g < kGroups; g += 32) {
      const int blk = g >> 3;
      const int i = min(blast, static_cast<int>((static_cast<float>(blk) + 0.5f) * stride_b) & ~31) + 4 * (g & 7);
      const uint32_t mb = static_cast<uint32_t>(static_cast<uint16_t>(__ldg(mrow + (i >> 4)))) >> (i & 15);
      float f[4];
      if constexpr (kVec) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(vals + i));
        f[0] = q.x; f[1] = q.y; f[2] = q.z; f[3] = q.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) f[e] = __ldg(vals + i + e);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t k = ((mb >> e) & 1u) ? key_of(f[e]) : kZeroKey;
        ks[4 * g + e] = k;
        kmax = k > kmax ? k : kmax;
        kmin = k < kmin ? k : kmin;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
      kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
    }
    // the r_lo-th largest key: a radix select over u = key - kmin, 8-bit digits from the top bit
    // of kmax - kmin (digits of the raw key put nearly every sample of a row in one or two bins)
    const uint32_t span = kmax - kmin;
    const int d = span ? 31 - __clz(span) : 0;
    uint32_t pre = 0u;
    int need = r_lo;
    int* h = sm.h[w];
    for (int s = d - 7;; s -= 8) {
      const int sh = s > 0 ? s : 0;
      const int nb = s + 8 - sh;
      const uint32_t dm = (1u << nb) - 1u;
      for (int i = lane; i < 256; i += 32) h[i] = 0;
      __syncwarp();
      for (int j = lane; j < kListSamples; j += 32) {
        const uint32_t u = ks[j] - kmin;
        if ((static_cast<uint64_t>(u) >> (sh + nb)) == pre) atomicAdd(&h[(u >> sh) & dm], 1);
      }
      __syncwarp();
      warp_find<256>(h, need, sm.res[w]);
      __syncwarp();
      pre = (pre << nb) | static_cast<uint32_t>(sm.res[w][0]);
      need -= sm.res[w][1];
      __syncwarp();
      if (sh == 0) break;
    }
    v = kmin + pre;
  }
  if (lane == 0) bounds[row] = static_cast<int32_t>(v ^ kZeroKey);
}

template <bool kVec>
__global__ __launch_bounds__(256) void list_collect_kernel(
    const float* __restrict__ score, int64_t score_stride, int width, const int16_t* __restrict__ mask,
    int64_t mask_stride, const int32_t* __restrict__ lengths, const int32_t* __restrict__ bounds, int rows,
    int2* __restrict__ lists, int cap, int32_t* __restrict__ cnt) {
  __shared__ __align__(16) uint32_t stage[256 * kLaneTok];  // each lane's 16 words of the current chunk
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int warp_in_cta = threadIdx.x >> 5;
  const int n_warps = static_cast<int>((gridDim.x * blockDim.x) >> 5);
  for (int row = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5); row < rows; row += n_warps) {
    int len = __ldg(lengths + row);
    len = len < 0 ? 0 : (len > width ? width : len);
    if (len <= kTopK) {  // the select writes these rows as the identity
      if (lane == 0) cnt[row] = 0;
      continue;
    }
    const uint32_t lo = len <= kListAllLen ? 0u : static_cast<uint32_t>(__ldg(bounds + row)) ^ kZeroKey;
    // a positive bound: a token passes iff its mask bit is set and its raw bits, as a signed int,
    // reach the bound's (the key order of positive floats), and its key is bits | sign bit
    const bool pos = lo > kZeroKey;
    const int lo_bits = static_cast<int>(lo & 0x7FFFFFFFu);
    const float* vals = score + static_cast<int64_t>(row) * score_stride;
    const int16_t* mrow = mask + static_cast<int64_t>(row) * mask_stride;
    int2* lst = lists + static_cast<int64_t>(row) * cap;
    int base = 0;  // uniform over the warp
    constexpr int kStep = 2 * 32 * kLaneTok;  // tokens per warp iteration (4 KB of scores)
    // the first two iterations' lines into L2, then each iteration prefetches the one two ahead:
    // the loads that follow find their lines in L2 (no registers held for the prefetch)
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int p = q * kStep + lane * 2 * kLaneTok;
      if (p < len) asm volatile("prefetch.global.L2 [%0];" ::"l"(vals + p));
    }
    for (int c0 = 0; c0 < len; c0 += kStep) {
      {
        const int p = c0 + 2 * kStep + lane * 2 * kLaneTok;  // 128 bytes per lane
        if (p < len) asm volatile("prefetch.global.L2 [%0];" ::"l"(vals + p));
      }
      uint32_t b[2][16], valid[2], mw[2];
#pragma unroll
      for (int u = 0; u < 2; ++u)
        mw[u] = load16_raw<kVec>(vals, mrow, c0 + (u * 32 + lane) * kLaneTok, len, b[u], valid[u]);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i0 = c0 + (u * 32 + lane) * kLaneTok;
        uint32_t hit = 0u;
        if (pos) {
#pragma unroll
          for (int e = 0; e < 16; ++e) hit |= (static_cast<int>(b[u][e]) >= lo_bits ? 1u : 0u) << e;
          hit &= mw[u] & valid[u];
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const uint32_t k = ((mw[u] >> e) & 1u) ? key_of(__uint_as_float(b[u][e])) : kZeroKey;
            b[u][e] = k;
            hit |= (((valid[u] >> e) & 1u) && k >= lo) ? (1u << e) : 0u;
          }
        }
        const int c = __popc(hit);
        const int inc = warp_incl_scan(c);
        int at = base + inc - c;
        base += __shfl_sync(0xffffffffu, inc, 31);
        if (hit) {  // the lane's words through shared memory, read back at the set bits only
          uint4* st4 = reinterpret_cast<uint4*>(stage + (warp_in_cta * 32 + lane) * kLaneTok);
#pragma unroll
          for (int q = 0; q < 4; ++q) st4[q] = make_uint4(b[u][4 * q], b[u][4 * q + 1], b[u][4 * q + 2], b[u][4 * q + 3]);
          const uint32_t* sw = stage + (warp_in_cta * 32 + lane) * kLaneTok;
          const uint32_t kbit = pos ? kZeroKey : 0u;
          do {
            const int e = __ffs(hit) - 1;
            hit &= hit - 1u;
            if (at < cap) lst[at] = make_int2(static_cast<int>(sw[e] | kbit), i0 + e);
            ++at;
          } while (hit);
        }
      }
    }
    if (lane == 0) cnt[row] = base;
  }
}

}  // namespace

// Used by the logits translation unit for the hist_lens path: zeroes the
// pass-1 workspace and preloads each row's +0 bin and zero count with its
// histogram length; the logits kernel's epilogue then does pass 1.
// Launchers of the fused prefill top-k (fused.cu): the list select, the exact
// top-k predicated on the select's flag, and the sampled per-row bound.
int launch_list_select(const int2* cand, const int32_t* cnt, int cap, const int32_t* row_end, int64_t rows,
                       int64_t width, const int32_t* bounds, int all_len, const int32_t* pt, int64_t pt_stride,
                       int32_t* dst, int32_t* flag, cudaStream_t stream, bool flag_per_row);

int launch_fused_select(const int2* cand, const int32_t* cnt, int cap, const int32_t* row_end, int64_t rows,
                        int64_t width, const int32_t* bounds, int all_len, const int32_t* pt, int64_t pt_stride,
                        int32_t* dst, int32_t* flag, cudaStream_t stream) {
  return launch_list_select(cand, cnt, cap, row_end, rows, width, bounds, all_len, pt, pt_stride, dst, flag, stream,
                            false);
}

int launch_list_select(const int2* cand, const int32_t* cnt, int cap, const int32_t* row_end, int64_t rows,
                       int64_t width, const int32_t* bounds, int all_len, const int32_t* pt, int64_t pt_stride,
                       int32_t* dst, int32_t* flag, cudaStream_t stream, bool flag_per_row) {
  if (rows <= 0) return HCU_OK;
  if (width > kFusedMaxWidth || cap > kFusedCap) return HCU_ERR_ARG;
  constexpr int kT = 256;
  const size_t smem = offsetof(FusedSelSmem<kT>, bm) + 2 * static_cast<size_t>((width + 31) / 32) * 4;
  cudaFuncSetAttribute(fused_select_kernel<kT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(sizeof(FusedSelSmem<kT>) + 2 * (kFusedMaxWidth / 32) * 4));
  fused_select_kernel<kT><<<static_cast<unsigned>(rows), kT, smem, stream>>>(
      cand, cnt, cap, row_end, static_cast<int>(width), bounds, all_len, pt, pt_stride, dst, flag,
      flag_per_row ? 1 : 0);
  return launch_status();
}

int launch_topk_if(const float* score, int64_t rows, int64_t width, int64_t score_stride, const int16_t* mask,
                   int64_t mask_stride, const int32_t* lengths, const int32_t* pt, int64_t pt_stride, int32_t* dst,
                   const int32_t* run_if, cudaStream_t stream) {
  if (rows <= 0) return HCU_OK;
  return launch_rows(score, rows, width, score_stride, mask, mask_stride, lengths, pt, pt_stride, dst, nullptr,
                     nullptr, stream, false, 1, run_if);
}

int launch_fused_bound(const float* score, int64_t score_stride, const int16_t* mask, int64_t mask_stride,
                       const int32_t* e_s, const int32_t* row_end, int64_t width, int64_t rows, int32_t* bounds,
                       cudaStream_t stream) {
  if (rows <= 0) return HCU_OK;
  const size_t smem = sizeof(FusedBoundSmem);
  cudaFuncSetAttribute(fused_bound_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  const unsigned grid = static_cast<unsigned>((rows + kFusedBoundWarps - 1) / kFusedBoundWarps);
  fused_bound_kernel<<<grid, kFusedBoundWarps * 32, smem, stream>>>(score, score_stride, mask, mask_stride, e_s,
                                                                     row_end, static_cast<int>(width),
                                                                     static_cast<int>(rows), bounds);
  return launch_status();
}

int fused_max_width() { return kFusedMaxWidth; }
int fused_max_cap() { return kFusedCap; }

int launch_hist_init(int32_t* zws, const int32_t* hist_lens, int64_t rows, int64_t width, cudaStream_t stream) {
  if (rows == 0) return HCU_OK;
  hist_init_kernel<<<static_cast<int>(rows), 256, 0, stream>>>(zws, hist_lens, static_cast<int>(width),
                                                              static_cast<int>(rows));
  return launch_status();
}

}  // namespace hcu

extern "C" int64_t hcu_topk_hist_ws_elems(int64_t rows) { return rows * (2 * hcu::kBins + 2); }

extern "C" int64_t hcu_topk_workspace_bytes(int64_t rows, int64_t width, int64_t max_splits) {
  (void)rows;
  (void)width;
  (void)max_splits;
  return 0;  // the single-CTA-per-row kernel keeps all state in shared memory
}

extern "C" int hcu_sparse_mask_topk_transform(const float* score, int64_t rows, int64_t width, int64_t score_stride,
                                              const int16_t* mask, int64_t mask_stride, const int32_t* lengths,
                                              const int32_t* page_table, int64_t pt_stride, int64_t topk,
                                              int32_t* dst, hcu_stream_t stream) {
  using namespace hcu;
  int st = check_common(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, topk,
                        dst);
  if (st != HCU_OK || rows == 0) return st;
  return launch_rows(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, dst,
                     nullptr, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

namespace hcu {
namespace {

struct ListLayout {
  int64_t bounds, cnt, fail, lists, total;
};

ListLayout list_layout(int64_t rows) {
  auto al = [](int64_t x) { return (x + 255) / 256 * 256; };
  ListLayout L{};
  int64_t o = 0;
  L.bounds = o;
  o += al(rows * 4);
  L.cnt = o;
  o += al(rows * 4);
  L.fail = o;
  o += al(rows * 4);
  L.lists = o;
  o += al(rows * static_cast<int64_t>(kFusedCap) * 8);
  L.total = o;
  return L;
}

}  // namespace
}  // namespace hcu

extern "C" int64_t hcu_sparse_mask_topk_transform_lists_workspace_bytes(int64_t rows, int64_t width) {
  if (rows < 0 || width < 0) return -1;
  return hcu::list_layout(rows).total;
}

extern "C" int hcu_sparse_mask_topk_transform_lists(const float* score, int64_t rows, int64_t width,
                                                    int64_t score_stride, const int16_t* mask, int64_t mask_stride,
                                                    const int32_t* lengths, const int32_t* page_table,
                                                    int64_t pt_stride, int64_t topk, void* workspace,
                                                    int64_t workspace_bytes, int32_t* dst, hcu_stream_t stream) {
  using namespace hcu;
  int st = check_common(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, topk,
                        dst);
  if (st != HCU_OK || rows == 0) return st;
  if (width > kFusedMaxWidth) return HCU_ERR_ARG;
  const ListLayout L = list_layout(rows);
  if (!workspace || workspace_bytes < L.total || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return HCU_ERR_ARG;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* bounds = reinterpret_cast<int32_t*>(ws + L.bounds);
  int32_t* cnt = reinterpret_cast<int32_t*>(ws + L.cnt);
  int32_t* fail = reinterpret_cast<int32_t*>(ws + L.fail);
  int2* lists = reinterpret_cast<int2*>(ws + L.lists);
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int w = static_cast<int>(width);
  const int r = static_cast<int>(rows);
  const bool vec = use_vec(score, width, score_stride);
  // the bound and the stream with programmatic stream serialization (each waits for the previous
  // kernel before its first read)
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const size_t bsmem = sizeof(ListBoundSmem);
  cfg.gridDim = dim3(static_cast<unsigned>((rows + kListBoundWarps - 1) / kListBoundWarps));
  cfg.blockDim = dim3(kListBoundWarps * 32);
  cfg.dynamicSmemBytes = bsmem;
  if (vec) {
    cudaFuncSetAttribute(list_bound_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bsmem));
    cudaLaunchKernelEx(&cfg, list_bound_kernel<true>, score, score_stride, w, mask, mask_stride, lengths, r, bounds);
  } else {
    cudaFuncSetAttribute(list_bound_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(bsmem));
    cudaLaunchKernelEx(&cfg, list_bound_kernel<false>, score, score_stride, w, mask, mask_stride, lengths, r, bounds);
  }
  if ((st = launch_status()) != HCU_OK) return st;
  cfg.gridDim = dim3(static_cast<unsigned>((rows + 7) / 8));  // one warp per row
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  if (vec)
    cudaLaunchKernelEx(&cfg, list_collect_kernel<true>, score, score_stride, w, mask, mask_stride, lengths,
                       static_cast<const int32_t*>(bounds), r, lists, kFusedCap, cnt);
  else
    cudaLaunchKernelEx(&cfg, list_collect_kernel<false>, score, score_stride, w, mask, mask_stride, lengths,
                       static_cast<const int32_t*>(bounds), r, lists, kFusedCap, cnt);
  if ((st = launch_status()) != HCU_OK) return st;
  if ((st = launch_list_select(lists, cnt, kFusedCap, lengths, rows, width, bounds, kListAllLen, page_table,
                               pt_stride, dst, fail, s, true)) != HCU_OK)
    return st;
  // rows whose list could not prove exactness: the block-per-row kernel, predicated per row
  return launch_rows(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, dst, nullptr,
                     nullptr, s, false, 1, fail, 1);
}

extern "C" int hcu_sparse_mask_topk_transform_split(const float* score, int64_t rows, int64_t width,
                                                    int64_t score_stride, const int16_t* mask, int64_t mask_stride,
                                                    const int32_t* lengths, const int32_t* page_table,
                                                    int64_t pt_stride, int64_t topk, int64_t max_splits,
                                                    void* workspace, int64_t workspace_bytes, int32_t* dst,
                                                    hcu_stream_t stream) {
  using namespace hcu;
  (void)workspace;
  (void)workspace_bytes;
  if (max_splits < 1) return HCU_ERR_ARG;
  int st = check_common(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, topk,
                        dst);
  if (st != HCU_OK || rows == 0) return st;
  return launch_rows(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, dst,
                     nullptr, nullptr, reinterpret_cast<cudaStream_t>(stream), false,
                     split_count(rows, width, max_splits));
}

extern "C" int hcu_sparse_mask_topk_transform_split_pre(const float* score, int64_t rows, int64_t width,
                                                        int64_t score_stride, const int16_t* mask,
                                                        int64_t mask_stride, const int32_t* lengths,
                                                        const int32_t* page_table, int64_t pt_stride, int64_t topk,
                                                        int64_t max_splits, int32_t* zws, void* workspace,
                                                        int64_t workspace_bytes, int32_t* dst,
                                                        hcu_stream_t stream) {
  using namespace hcu;
  (void)workspace;
  (void)workspace_bytes;
  if (max_splits < 1 || zws == nullptr) return HCU_ERR_ARG;
  int st = check_common(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, topk,
                        dst);
  if (st != HCU_OK || rows == 0) return st;
  return launch_rows(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, dst,
                     nullptr, zws, reinterpret_cast<cudaStream_t>(stream), false, split_count(rows, width, max_splits));
}

extern "C" int hcu_topk_keys(const float* score, int64_t rows, int64_t width, int64_t score_stride,
                             const int16_t* mask, int64_t mask_stride, const int32_t* lengths,
                             const int32_t* page_table, int64_t pt_stride, int32_t* dst, uint32_t* dst_keys,
                             hcu_stream_t stream) {
  using namespace hcu;
  int st = check_common(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, kTopK,
                        dst);
  if (st != HCU_OK || rows == 0) return st;
  if (!dst_keys) return HCU_ERR_ARG;
  return launch_rows(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, dst,
                     dst_keys, nullptr, reinterpret_cast<cudaStream_t>(stream), /*sorted=*/true);
}

extern "C" int hcu_topk_keys_if(const float* score, int64_t rows, int64_t width, int64_t score_stride,
                                const int16_t* mask, int64_t mask_stride, const int32_t* lengths,
                                const int32_t* page_table, int64_t pt_stride, int32_t* dst, uint32_t* dst_keys,
                                const int32_t* run_if, hcu_stream_t stream) {
  using namespace hcu;
  int st = check_common(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, kTopK,
                        dst);
  if (st != HCU_OK || rows == 0) return st;
  if (!dst_keys || !run_if) return HCU_ERR_ARG;
  return launch_rows(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, dst,
                     dst_keys, nullptr, reinterpret_cast<cudaStream_t>(stream), /*sorted=*/true, 1, run_if);
}

extern "C" int hcu_cp_topk_merge_lists(const uint32_t* keys, const int32_t* gidx, int64_t n_parts,
                                       int64_t list_len, int64_t part_stride, int64_t rows, const int32_t* lengths,
                                       int32_t* flag, int32_t short_identity, int32_t* dst, hcu_stream_t stream) {
  using namespace hcu;
  if (n_parts < 1 || n_parts > kMaxParts || rows < 0 || rows > INT32_MAX) return HCU_ERR_ARG;
  if (part_stride < rows * list_len) return HCU_ERR_ARG;
  int lshift = 0;
  while ((int64_t{1} << lshift) < list_len) ++lshift;
  if ((int64_t{1} << lshift) != list_len || list_len < 256 || list_len > kTopK || n_parts * list_len < kTopK)
    return HCU_ERR_ARG;
  if (rows == 0) return HCU_OK;
  if (!keys || !gidx || !lengths || !dst) return HCU_ERR_ARG;
  // one 1024-thread CTA per row (a 512-thread instance, two CTAs per SM, measured slower: its
  // 4096-entry candidate list overflows into the exact fallback on the bounded exchange's lists)
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t smem = sizeof(TopkSmem<1024>);
  cudaFuncSetAttribute(cp_merge_kernel<1024>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  cp_merge_kernel<1024><<<static_cast<unsigned>(rows), 1024, smem, st>>>(
      keys, gidx, static_cast<int>(n_parts), lshift, part_stride, lengths, dst, flag, short_identity);
  return launch_status();
}

extern "C" int hcu_cp_topk_merge(const uint32_t* keys, const int32_t* gidx, int64_t n_parts, int64_t rows,
                                 const int32_t* lengths, int32_t* dst, hcu_stream_t stream) {
  return hcu_cp_topk_merge_lists(keys, gidx, n_parts, hcu::kTopK, rows * hcu::kTopK, rows, lengths, nullptr, 0, dst,
                                 stream);
}

extern "C" int hcu_cp_local_bound(const float* score, int64_t rows, int64_t width, int64_t score_stride,
                                  const int16_t* mask, int64_t mask_stride, const int32_t* lengths,
                                  const int32_t* totals, int32_t* bounds, hcu_stream_t stream) {
  using namespace hcu;
  if (rows < 0 || rows > INT32_MAX || width < 0 || width > INT32_MAX / 2) return HCU_ERR_ARG;
  if (rows == 0) return HCU_OK;
  if (!score || !mask || !lengths || !totals || !bounds) return HCU_ERR_ARG;
  if (score_stride < width || mask_stride < (width + 15) / 16) return HCU_ERR_ARG;
  const size_t smem = sizeof(BoundSmem);
  const unsigned grid = static_cast<unsigned>((rows + kBoundWarps - 1) / kBoundWarps);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (use_vec(score, width, score_stride)) {
    cudaFuncSetAttribute(cp_bound_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    cp_bound_kernel<true><<<grid, kBoundWarps * 32, smem, st>>>(score, score_stride, static_cast<int>(width), mask,
                                                                mask_stride, lengths, totals, static_cast<int>(rows),
                                                                bounds);
  } else {
    cudaFuncSetAttribute(cp_bound_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    cp_bound_kernel<false><<<grid, kBoundWarps * 32, smem, st>>>(score, score_stride, static_cast<int>(width), mask,
                                                                 mask_stride, lengths, totals, static_cast<int>(rows),
                                                                 bounds);
  }
  return launch_status();
}

namespace hcu {
namespace {
template <int kT, bool kVec>
void launch_filter(const float* score, int rows, int width, int64_t score_stride, const int16_t* mask,
                   int64_t mask_stride, const int32_t* lengths, const int32_t* pt, int64_t pt_stride,
                   const int32_t* bounds, int cap, uint32_t* keys, int32_t* gidx, int rpb, int64_t bstride,
                   int32_t* counts, int32_t* flag, cudaStream_t st) {
  const size_t smem = sizeof(TopkSmem<kT>);
  cudaFuncSetAttribute(cp_filter_kernel<kT, kVec>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  // persistent CTAs; the warp pass when this CTA's rows fit its overflow bitmap
  const int grid = static_cast<int>(std::min<int64_t>(rows, static_cast<int64_t>(sm_count()) * (1024 / kT)));
  const int warp_pass = (rows + grid - 1) / grid <= kFilterRowsPerCta ? 1 : 0;
  cp_filter_kernel<kT, kVec><<<static_cast<unsigned>(grid), kT, smem, st>>>(
      score, score_stride, width, mask, mask_stride, lengths, pt, pt_stride, bounds, cap, keys, gidx, rpb, bstride,
      counts, flag, rows, warp_pass);
}
}  // namespace
}  // namespace hcu

extern "C" int hcu_cp_filter(const float* score, int64_t rows, int64_t width, int64_t score_stride,
                             const int16_t* mask, int64_t mask_stride, const int32_t* lengths,
                             const int32_t* page_table, int64_t pt_stride, const int32_t* bounds, int64_t cap,
                             uint32_t* keys, int32_t* gidx, int64_t rows_per_block, int64_t block_stride,
                             int32_t* counts, int32_t* flag, hcu_stream_t stream) {
  using namespace hcu;
  int st = check_common(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, kTopK,
                        gidx);
  if (st != HCU_OK || rows == 0) return st;
  if (!bounds || !keys || !flag || cap < 1 || cap > kTopK) return HCU_ERR_ARG;
  if (rows_per_block < 1 || rows_per_block > INT32_MAX ||
      (rows > rows_per_block && block_stride < rows_per_block * cap))
    return HCU_ERR_ARG;
  const int r = static_cast<int>(rows), w = static_cast<int>(width), c = static_cast<int>(cap);
  const int rpb = static_cast<int>(rows_per_block);
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = use_vec(score, width, score_stride);
  if (width <= kNarrowWidth || (rows >= 2 * static_cast<int64_t>(sm_count()) && width <= kManyRowsWidth)) {
    if (vec)
      launch_filter<512, true>(score, r, w, score_stride, mask, mask_stride, lengths, page_table, pt_stride, bounds, c,
                               keys, gidx, rpb, block_stride, counts, flag, s);
    else
      launch_filter<512, false>(score, r, w, score_stride, mask, mask_stride, lengths, page_table, pt_stride, bounds,
                                c, keys, gidx, rpb, block_stride, counts, flag, s);
  } else {
    if (vec)
      launch_filter<1024, true>(score, r, w, score_stride, mask, mask_stride, lengths, page_table, pt_stride, bounds,
                                c, keys, gidx, rpb, block_stride, counts, flag, s);
    else
      launch_filter<1024, false>(score, r, w, score_stride, mask, mask_stride, lengths, page_table, pt_stride, bounds,
                                 c, keys, gidx, rpb, block_stride, counts, flag, s);
  }
  return launch_status();
}

// ---------------------------------------------------------------------------
// Context-parallel exchange over peer memory (hcu_cp_peer_*): the bound, filter
// and merge kernels store their results straight into the consuming ranks'
// buffers (mapped over NVLink) and publish completion with one flag per (step,
// phase, source rank); the consumers wait for every rank's flag.
//
// Publication: the CTA synchronises, thread 0 fences the CTA's stores at
// system scope and counts the CTA into a local counter; the launch's
// last CTA (it sees the count reach the grid size) resets the counter, takes
// the launch's local flag word and stores (epoch << 1 | flag) into every
// rank's signal word for (phase, this rank) with a system-scope release.
// Waiting: thread 0 spins with acquire loads on the P words of the phase until
// each holds this epoch, bounded by the wait limit (on expiry the status bit is
// set and the CTA skips its work, flagging the step); the CTA then synchronises.
// ---------------------------------------------------------------------------
namespace hcu {
namespace {

enum : int {
  kWsBoundCnt = 0, kWsFilterCnt = 1, kWsMergeCnt = 2, kWsScatterCnt = 3, kWsXMergeCnt = 4,
  kWsFilterFlag = 5, kWsMergeFlag = 6, kWsXMergeFlag = 7,
};
enum : int { kPhBounds = 0, kPhLists = 1, kPhRows = 2, kPhXLists = 3, kPhXRows = 4 };
static_assert(HCU_CP_SIG_WORDS == 5 && HCU_CP_WS_FLAG == 8 && HCU_CP_WS_RERUNS == 9, "signal and workspace layout");

__device__ __forceinline__ void peer_publish(const hcu_cp_peers_t& pp, int phase, int* counter, int* flagw) {
  // The CTA barrier orders every thread's stores before thread 0's system-scope fence, whose
  // release is cumulative over them (the pattern of a grid-wide barrier): one fence per CTA
  // instead of one per thread.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int grid = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(reinterpret_cast<unsigned int*>(counter), 1u) + 1u == grid) {
      __threadfence_system();
      const int f = flagw ? atomicExch(flagw, 0) : 0;
      atomicExch(counter, 0);
      const uint32_t v = (pp.epoch << 1) | (f != 0 ? 1u : 0u);
      for (int p = 0; p < pp.parts; ++p) st_release_sys(pp.sig[p] + phase * pp.parts + pp.rank, v);
    }
  }
}

// Thread 0 only.  True when every rank published `phase` for this epoch; *flag
// = the OR of their flag bits.  False (status set) when the wait limit passed.
__device__ __noinline__ bool peer_wait(const hcu_cp_peers_t& pp, int phase, int* flag) {
  const uint32_t* sig = pp.sig[pp.rank] + phase * pp.parts;
  const uint64_t lim = wait_limit_ns();
  const uint64_t t0 = globaltimer();
  int f = 0;
  for (int p = 0; p < pp.parts; ++p) {
    uint32_t v = ld_acquire_sys(sig + p);
    while ((v >> 1) < pp.epoch) {
      if (globaltimer() - t0 > lim) {
        atomicOr(&g_hcu_status, HCU_STATUS_WAIT_TIMEOUT);
        *flag = 1;
        return false;
      }
      __nanosleep(128);
      v = ld_acquire_sys(sig + p);
    }
    f |= static_cast<int>(v & 1u);
  }
  *flag = f;
  return true;
}

// Waits in thread 0 and shares the outcome with the CTA; the flag bits of the
// sources are ORed into *flagw (when given).
__device__ __forceinline__ bool cta_wait(const hcu_cp_peers_t& pp, int phase, int* flagw, int* s_ok) {
  if (threadIdx.x == 0) {
    int f = 0;
    *s_ok = peer_wait(pp, phase, &f) ? 1 : 0;
    if (f && flagw) atomicOr(flagw, 1);
  }
  __syncthreads();
  return *s_ok != 0;
}

template <bool kVec>
__global__ __launch_bounds__(kBoundWarps * 32) void cp_peer_bound_kernel(
    const float* __restrict__ score, int64_t score_stride, int width, const int16_t* __restrict__ mask,
    int64_t mask_stride, const int32_t* __restrict__ lengths, const int32_t* __restrict__ totals,
    const hcu_cp_peers_t pp) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BoundSmem& sm = *reinterpret_cast<BoundSmem*>(smem_raw);
  __shared__ __align__(16) int32_t vals[kBoundWarps];
  const int w = threadIdx.x >> 5;
  const int row0 = blockIdx.x * kBoundWarps;
  const int row = row0 + w;
  if (row < pp.rows) {
    const uint32_t v = row_bound<kVec>(sm, score, score_stride, width, mask, mask_stride, lengths, totals, row);
    if ((threadIdx.x & 31) == 0) vals[w] = static_cast<int32_t>(v ^ kZeroKey);
  }
  __syncthreads();
  // the CTA's (up to) 8 consecutive bounds into slot `rank` of every rank's [P, R] bounds
  const int nv = min(kBoundWarps, pp.rows - row0);
  for (int i = threadIdx.x; i < pp.parts * nv; i += blockDim.x) {
    const int p = i / nv, j = i - (i / nv) * nv;
    pp.bounds[p][static_cast<int64_t>(pp.rank) * pp.rows + row0 + j] = vals[j];
  }
  peer_publish(pp, kPhBounds, pp.ws + kWsBoundCnt, nullptr);
}

template <int kT, bool kVec>
__global__ __launch_bounds__(kT, 1024 / kT) void cp_peer_filter_kernel(
    const float* __restrict__ score, int64_t score_stride, int width, const int16_t* __restrict__ mask,
    int64_t mask_stride, const int32_t* __restrict__ lengths, const int32_t* __restrict__ pt, int64_t pt_stride,
    const hcu_cp_peers_t pp, int warp_pass) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TopkSmem<kT>& sm = *reinterpret_cast<TopkSmem<kT>*>(smem_raw);
  __shared__ int s_ok;
  __shared__ uint32_t ovf[kFilterRowsPerCta / 32];  // rows (by their index in this CTA) left to filter_row
  int* flagw = pp.ws + kWsFilterFlag;
  // the row's bound: the minimum over ranks of their published estimates (order-preserving int32)
  auto lo_of = [&](int row) {
    int32_t b = INT32_MAX;
    const int32_t* bl = pp.bounds[pp.rank];
    for (int p = 0; p < pp.parts; ++p) b = min(b, __ldcg(bl + static_cast<int64_t>(p) * pp.rows + row));
    return static_cast<uint32_t>(b) ^ kZeroKey;
  };
  auto len_of = [&](int row) {
    const int len = __ldg(lengths + row);
    return len < 0 ? 0 : (len > width ? width : len);
  };
  // this rank's list of the row in its owner's buffer: keys, then (rows_per_rank * C later) entries
  auto keys_of = [&](int row) {
    return pp.lists[row / pp.rows_per_rank] +
           (static_cast<int64_t>(2 * pp.rank) * pp.rows_per_rank + row % pp.rows_per_rank) * pp.list_len;
  };
  const int64_t ent = static_cast<int64_t>(pp.rows_per_rank) * pp.list_len;
  // persistent CTAs (rows strided over the grid): one wait and one publication per CTA; with
  // warp_pass, first a warp per row, then the CTA on the rows whose list overflowed
  if (cta_wait(pp, kPhBounds, nullptr, &s_ok)) {
    const int nk =
        (pp.rows - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
    if (warp_pass) {
      for (int i = threadIdx.x; i < kFilterRowsPerCta / 32; i += kT) ovf[i] = 0u;
      __syncthreads();
      const int w = threadIdx.x >> 5;
      uint32_t* stage = reinterpret_cast<uint32_t*>(&sm.scr[0][0]) + w * 32 * kLaneTok;
      for (int k = w; k < nk; k += kT / 32) {
        const int row = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
        int32_t* keys = keys_of(row);
        const int n = filter_row_warp<kVec>(score + static_cast<int64_t>(row) * score_stride,
                                            mask + static_cast<int64_t>(row) * mask_stride,
                                            pt + static_cast<int64_t>(row) * pt_stride, len_of(row), lo_of(row),
                                            pp.list_len, reinterpret_cast<uint32_t*>(keys), keys + ent, stage);
        if ((threadIdx.x & 31) == 0 && n > pp.list_len) atomicOr(&ovf[k >> 5], 1u << (k & 31));
      }
      __syncthreads();
    }
    for (int k = 0; k < nk; ++k) {
      if (warp_pass && !((ovf[k >> 5] >> (k & 31)) & 1u)) continue;  // uniform: shared state
      const int row = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
      int32_t* keys = keys_of(row);
      filter_row<kT, kVec>(sm, score + static_cast<int64_t>(row) * score_stride,
                           mask + static_cast<int64_t>(row) * mask_stride, pt + static_cast<int64_t>(row) * pt_stride,
                           len_of(row), lo_of(row), pp.list_len, reinterpret_cast<uint32_t*>(keys), keys + ent,
                           flagw);
      __syncthreads();  // the row's shared state is read out before the next row reuses it
    }
  } else if (threadIdx.x == 0) {
    atomicOr(flagw, 1);
  }
  peer_publish(pp, kPhLists, pp.ws + kWsFilterCnt, flagw);
}

// Persistent CTAs over the rps rows of this rank: each waits once for every
// rank's lists of the step, then per row merges the lists into this rank's out
// row and copies that row to every other rank's out.  exact: the 2048-entry
// lists of the redo (predicated on the flag: with it clear the small grid
// returns at once).
template <int kT>
__global__ __launch_bounds__(kT, 1024 / kT) void cp_peer_merge_kernel(const int32_t* __restrict__ totals, int exact,
                                                                     const hcu_cp_peers_t pp) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TopkSmem<kT>& sm = *reinterpret_cast<TopkSmem<kT>*>(smem_raw);
  __shared__ int s_ok;
  if (exact && __ldcg(pp.ws + HCU_CP_WS_FLAG) == 0) return;  // grid-uniform: no redo this step
  const int rps = pp.rows_per_rank;
  int* flagw = pp.ws + (exact ? kWsXMergeFlag : kWsMergeFlag);
  // persistent CTAs (rows strided over the grid): one wait and one publication per CTA
  const bool ok = cta_wait(pp, exact ? kPhXLists : kPhLists, flagw, &s_ok);
  if (!ok && threadIdx.x == 0) atomicOr(flagw, 1);
  for (int row = blockIdx.x; row < rps; row += gridDim.x) {
    const int64_t off = (static_cast<int64_t>(pp.rank) * rps + row) * kTopK;
    int32_t* mine = pp.out[pp.rank] + off;
    if (ok) {
      const int C = exact ? kTopK : pp.list_len;
      const int lshift = 31 - __clz(C);
      const int32_t* lists = exact ? pp.lists_exact[pp.rank] : pp.lists[pp.rank];
      merge_row(sm, reinterpret_cast<const uint32_t*>(lists), lists + static_cast<int64_t>(rps) * C, pp.parts,
                lshift, 2 * static_cast<int64_t>(rps) * C, totals, row, mine, flagw, 1);
    }
    __syncthreads();  // the row is complete in this rank's out
    const int4* src = reinterpret_cast<const int4*>(mine);
    for (int i = threadIdx.x; i < kTopK / 4; i += kT) {
      const int4 v = __ldcg(src + i);
      for (int p = 0; p < pp.parts; ++p)
        if (p != pp.rank) reinterpret_cast<int4*>(pp.out[p] + off)[i] = v;
    }
    __syncthreads();  // shared state free for the next row
  }
  peer_publish(pp, exact ? kPhXRows : kPhRows, pp.ws + (exact ? kWsXMergeCnt : kWsMergeCnt), flagw);
}

// The redo's lists: row r's local top-2048 (keys, entries) into slot `rank` of its owner's lists_exact.
__global__ __launch_bounds__(256) void cp_peer_scatter_kernel(const uint32_t* __restrict__ keys,
                                                              const int32_t* __restrict__ entries,
                                                              const hcu_cp_peers_t pp) {
  if (__ldcg(pp.ws + HCU_CP_WS_FLAG) == 0) return;  // grid-uniform
  const int row = blockIdx.x;
  const int rps = pp.rows_per_rank;
  int32_t* dk = pp.lists_exact[row / rps] + (static_cast<int64_t>(2 * pp.rank) * rps + row % rps) * kTopK;
  int32_t* dg = dk + static_cast<int64_t>(rps) * kTopK;
  const int4* sk = reinterpret_cast<const int4*>(keys + static_cast<int64_t>(row) * kTopK);
  const int4* sg = reinterpret_cast<const int4*>(entries + static_cast<int64_t>(row) * kTopK);
  for (int i = threadIdx.x; i < kTopK / 4; i += blockDim.x) {
    reinterpret_cast<int4*>(dk)[i] = __ldcg(sk + i);
    reinterpret_cast<int4*>(dg)[i] = __ldcg(sg + i);
  }
  peer_publish(pp, kPhXLists, pp.ws + kWsScatterCnt, nullptr);
}

// Waits for every rank's rows of the step; the bounded pass records the step's
// flag (the OR over ranks, identical on every rank), the redo counts itself.
__global__ __launch_bounds__(32) void cp_peer_finish_kernel(int exact, const hcu_cp_peers_t pp) {
  if (threadIdx.x != 0) return;
  if (exact && __ldcg(pp.ws + HCU_CP_WS_FLAG) == 0) return;
  int f = 0;
  const bool ok = peer_wait(pp, exact ? kPhXRows : kPhRows, &f);
  if (!exact)
    atomicExch(pp.ws + HCU_CP_WS_FLAG, (f || !ok) ? 1 : 0);
  else
    atomicAdd(pp.ws + HCU_CP_WS_RERUNS, 1);
}

int check_peers(const hcu_cp_peers_t* pp) {
  if (!pp) return HCU_ERR_ARG;
  const hcu_cp_peers_t& p = *pp;
  if (p.parts < 1 || p.parts > HCU_CP_MAX_PARTS || p.rank < 0 || p.rank >= p.parts || p.rows < 0) return HCU_ERR_ARG;
  if (p.rows_per_rank < 0 || static_cast<int64_t>(p.rows_per_rank) * p.parts < p.rows) return HCU_ERR_ARG;
  if (p.list_len < 256 || p.list_len > kTopK || (p.list_len & (p.list_len - 1)) ||
      static_cast<int64_t>(p.list_len) * p.parts < kTopK)
    return HCU_ERR_ARG;
  if (p.epoch < 1 || p.epoch > 0x7FFFFFFFu || !p.ws) return HCU_ERR_ARG;
  for (int i = 0; i < p.parts; ++i)
    if (!p.bounds[i] || !p.lists[i] || !p.lists_exact[i] || !p.out[i] || !p.sig[i]) return HCU_ERR_ARG;
  return HCU_OK;
}

template <int kT, bool kVec>
void launch_peer_filter(const float* score, int width, int64_t score_stride, const int16_t* mask, int64_t mask_stride,
                        const int32_t* lengths, const int32_t* pt, int64_t pt_stride, const hcu_cp_peers_t& pp,
                        cudaStream_t st) {
  const size_t smem = sizeof(TopkSmem<kT>);
  cudaFuncSetAttribute(cp_peer_filter_kernel<kT, kVec>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  const int grid = static_cast<int>(std::min<int64_t>(pp.rows, static_cast<int64_t>(sm_count()) * (1024 / kT)));
  const int warp_pass = (pp.rows + grid - 1) / grid <= kFilterRowsPerCta ? 1 : 0;
  cp_peer_filter_kernel<kT, kVec><<<static_cast<unsigned>(grid), kT, smem, st>>>(
      score, score_stride, width, mask, mask_stride, lengths, pt, pt_stride, pp, warp_pass);
}

}  // namespace
}  // namespace hcu

extern "C" int hcu_cp_peer_bound(const float* score, int64_t width, int64_t score_stride, const int16_t* mask,
                                 int64_t mask_stride, const int32_t* lengths, const int32_t* totals,
                                 const hcu_cp_peers_t* peers, hcu_stream_t stream) {
  using namespace hcu;
  if (check_peers(peers) != HCU_OK) return HCU_ERR_ARG;
  const hcu_cp_peers_t& pp = *peers;
  if (width < 0 || width > INT32_MAX / 2 || score_stride < width || mask_stride < (width + 15) / 16) return HCU_ERR_ARG;
  if (pp.rows == 0) return HCU_OK;
  if (!score || !mask || !lengths || !totals) return HCU_ERR_ARG;
  const size_t smem = sizeof(BoundSmem);
  const unsigned grid = static_cast<unsigned>((pp.rows + kBoundWarps - 1) / kBoundWarps);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (use_vec(score, width, score_stride)) {
    cudaFuncSetAttribute(cp_peer_bound_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    cp_peer_bound_kernel<true><<<grid, kBoundWarps * 32, smem, st>>>(score, score_stride, static_cast<int>(width),
                                                                     mask, mask_stride, lengths, totals, pp);
  } else {
    cudaFuncSetAttribute(cp_peer_bound_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    cp_peer_bound_kernel<false><<<grid, kBoundWarps * 32, smem, st>>>(score, score_stride, static_cast<int>(width),
                                                                      mask, mask_stride, lengths, totals, pp);
  }
  return launch_status();
}

extern "C" int hcu_cp_peer_filter(const float* score, int64_t width, int64_t score_stride, const int16_t* mask,
                                  int64_t mask_stride, const int32_t* lengths, const int32_t* page_table,
                                  int64_t pt_stride, const hcu_cp_peers_t* peers, hcu_stream_t stream) {
  using namespace hcu;
  if (check_peers(peers) != HCU_OK) return HCU_ERR_ARG;
  const hcu_cp_peers_t& pp = *peers;
  const int st0 = check_common(score, pp.rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride,
                               kTopK, page_table);
  if (st0 != HCU_OK || pp.rows == 0) return st0;
  const int w = static_cast<int>(width);
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = use_vec(score, width, score_stride);
  if (width <= kNarrowWidth || (pp.rows >= 2 * static_cast<int64_t>(sm_count()) && width <= kManyRowsWidth)) {
    vec ? launch_peer_filter<512, true>(score, w, score_stride, mask, mask_stride, lengths, page_table, pt_stride, pp, s)
        : launch_peer_filter<512, false>(score, w, score_stride, mask, mask_stride, lengths, page_table, pt_stride, pp,
                                         s);
  } else {
    vec ? launch_peer_filter<1024, true>(score, w, score_stride, mask, mask_stride, lengths, page_table, pt_stride, pp,
                                         s)
        : launch_peer_filter<1024, false>(score, w, score_stride, mask, mask_stride, lengths, page_table, pt_stride,
                                          pp, s);
  }
  return launch_status();
}

extern "C" int hcu_cp_peer_merge(const int32_t* totals, int32_t exact, const hcu_cp_peers_t* peers,
                                 hcu_stream_t stream) {
  using namespace hcu;
  if (check_peers(peers) != HCU_OK || !totals) return HCU_ERR_ARG;
  const hcu_cp_peers_t& pp = *peers;
  if (pp.rows_per_rank == 0) return HCU_OK;
  const size_t smem = sizeof(TopkSmem<1024>);
  cudaFuncSetAttribute(cp_peer_merge_kernel<1024>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  const int grid = static_cast<int>(std::min<int64_t>(pp.rows_per_rank, sm_count()));
  cp_peer_merge_kernel<1024><<<static_cast<unsigned>(grid), 1024, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      totals, exact ? 1 : 0, pp);
  return launch_status();
}

extern "C" int hcu_cp_peer_scatter_exact(const uint32_t* keys, const int32_t* entries, const hcu_cp_peers_t* peers,
                                         hcu_stream_t stream) {
  using namespace hcu;
  if (check_peers(peers) != HCU_OK || !keys || !entries) return HCU_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(keys) | reinterpret_cast<uintptr_t>(entries)) % 16 != 0) return HCU_ERR_ARG;
  if (peers->rows == 0) return HCU_OK;
  cp_peer_scatter_kernel<<<static_cast<unsigned>(peers->rows), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      keys, entries, *peers);
  return launch_status();
}

extern "C" int hcu_cp_peer_finish(int32_t exact, const hcu_cp_peers_t* peers, hcu_stream_t stream) {
  using namespace hcu;
  if (check_peers(peers) != HCU_OK) return HCU_ERR_ARG;
  cp_peer_finish_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(exact ? 1 : 0, *peers);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Allocation-free top-k for callers that may not allocate device memory.
//
// The regular pass-1 path needs a workspace the caller allocates (zws, from
// hcu_mqa_logits_hist).  Some callers cannot allocate: code running inside an
// engine that owns the device memory pool, or a plug-in invoked where a
// cudaMalloc would synchronise the device or break the host's memory budget.
// This entry point keeps that workspace in one fixed file-scope device array
// (kNoAllocMaxRows rows, 8 MiB, held by every GPU that loads this library until
// the process exits) and otherwise runs the same kernels as the split_pre path.
// ---------------------------------------------------------------------------
namespace hcu {
namespace {

constexpr int64_t kNoAllocMaxRows = 256;

// pass-1 workspace [ghist1 rows*4096 | ghist2 rows*4096 | cnt rows*2] of one call
static __device__ __align__(256) int32_t g_topk_noalloc_ws[kNoAllocMaxRows * (2 * kBins + 2)];

// Device address of g_topk_noalloc_ws on the current device, looked up once per
// device (host code only holds a stand-in for the array under its name).
int32_t* noalloc_ws_address() {
  static std::mutex mu;
  static std::vector<int32_t*> cache;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_error(e);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, nullptr);
  if (cache[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_topk_noalloc_ws);
    if (e != cudaSuccess) {
      set_last_error(e);
      return nullptr;
    }
    cache[dev] = static_cast<int32_t*>(ptr);
  }
  return cache[dev];
}

}  // namespace
}  // namespace hcu

extern "C" int64_t hcu_topk_noalloc_max_rows(void) { return hcu::kNoAllocMaxRows; }

extern "C" int hcu_sparse_mask_topk_transform_noalloc(const float* score, int64_t rows, int64_t width,
                                                      int64_t score_stride, const int16_t* mask, int64_t mask_stride,
                                                      const int32_t* lengths, const int32_t* page_table,
                                                      int64_t pt_stride, int64_t topk, int32_t* dst,
                                                      hcu_stream_t stream) {
  using namespace hcu;
  int st = check_common(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, topk,
                        dst);
  if (st != HCU_OK || rows == 0) return st;
  if (rows > kNoAllocMaxRows) {
    set_last_error_msg("hcu_sparse_mask_topk_transform_noalloc: rows exceeds the fixed scratch maximum of ",
                       "256 rows (call the regular entry point for larger batches)");
    return HCU_ERR_ARG;
  }
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (width <= kTopK)  // every row is short (its first `len` page-table entries, -1 pads): no histogram needed
    return launch_rows(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, dst,
                       nullptr, nullptr, s);
  int32_t* ws = noalloc_ws_address();
  if (ws == nullptr) return HCU_ERR_LAUNCH;
  // hist_init_kernel rewrites every workspace element the later kernels read (the
  // array keeps the previous call's contents)
  hist_init_kernel<<<static_cast<int>(rows), 256, 0, s>>>(ws, lengths, static_cast<int>(width),
                                                          static_cast<int>(rows));
  const dim3 grid(static_cast<unsigned>((width + kHistChunk - 1) / kHistChunk), static_cast<unsigned>(rows));
  pass1_hist_kernel<<<grid, kHistThreads, 0, s>>>(score, score_stride, static_cast<int>(width), mask, mask_stride,
                                                 lengths, ws, static_cast<int>(rows));
  st = launch_status();
  if (st != HCU_OK) return st;
  return launch_rows(score, rows, width, score_stride, mask, mask_stride, lengths, page_table, pt_stride, dst,
                     nullptr, ws, s);
}
