// Stage 2: MQA index logits on the 5th-generation tensor cores (sm_100a).
//
//   s[row, t] = (sum_h w[row, h] * relu(q[row, h, :] . k[t, :])) * k_scale[t]
//
// Paged decode kernel (mqa_logits_paged_kernel), one persistent CTA per SM:
//   * the work list is (request group, row block, 128-token tile) flattened in
//     that order and cut into one contiguous range per CTA (balanced to one
//     tile; Q changes only at group boundaries).  It is derived on the device
//     from the context lengths, so the launch is CUDA-graph capturable;
//   * TMA producers (warp 0 and kProducers - 1 more warps, items dealt round
//     robin): per tile two 3-D TMA box loads {128 B, 64 tok, 1} of the two
//     64-token K pages named by the block table (128-byte swizzle, a K-major
//     UMMA operand) and their scale boxes, into an 8-stage ring;
//   * warp 1 (MMA issuer): loads each row block's R*H Q rows (2-D TMA, two
//     slots), then tcgen05.mma.cta_group::1.kind::f8f6f4, M = 128 tokens,
//     N = R*H query heads, K = 128 as 4 x 32, accumulating fp32 in 4 TMEM
//     buffers (2 when N > 128); tcgen05.commit frees the stage and publishes
//     the accumulator;
//   * epilogue (kTeams teams of 4 warps, one per TMEM lane quadrant, taking
//     tiles round robin): thread = token = TMEM lane; tcgen05.ld of the row's
//     H columns, ReLU * w head sum in registers, * k_scale, mask bit via warp
//     ballot, logits stored only where the bit is set; with hist_lens the
//     same epilogue does pass 1 of the top-k (key[31:20] bins, +0 and
//     positive counts) with global atomics into the workspace (kHist).
// Semantics follow hcu_ops/csrc/mqa_hist.cu:97-273 of the reference: lengths
// clamped to [0, width], every row of a group reads the group's first block
// table row, mask bit = token < len && bits(s) != 0.
//
// Every mbarrier wait is bounded (common.cuh); on expiry the CTA records
// HCU_STATUS_WAIT_TIMEOUT, stops issuing, drains the copies and MMAs it issued
// and frees its TMEM before returning.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "common.cuh"

HCU_DEFINE_STATUS(status_logits)

namespace hcu {
int launch_hist_init(int32_t* zws, const int32_t* hist_lens, int64_t rows, int64_t width, cudaStream_t stream);

namespace {

constexpr int kTeams = 3;        // epilogue teams of 4 warps (one per TMEM lane quadrant) on alternate tiles
constexpr int kEpiWarps = 4 * kTeams;
constexpr int kProducers = 4;  // TMA producer warps; producer k issues every box of the items it % kProducers == k
constexpr int kProducerB = 2 + kEpiWarps;  // first of the extra TMA producer warps
constexpr int kLgThreads = (2 + kEpiWarps + kProducers - 1) * 32;  // warp 0 + extra TMA, warp 1 MMA, 2.. epilogue
// Above 16 warps a thread has at most 96 registers: the epilogue then reads one
// 32-head TMEM chunk at a time instead of a whole row.
constexpr bool kPgChunked = kLgThreads > 512;
constexpr int kMaxAcc = 4;     // TMEM accumulator buffers (4 when N <= 128, else 2)
constexpr int kStages = 8;       // K-tile stages when a row block spans more than 128 TMEM columns
constexpr int kStagesNarrow = 8;   // stages when it spans <= 128 (room for 10 with 16 KB Q slots; 10 measured slower)
constexpr int kTileTok = 128;
constexpr int kATile = kTileTok * kHeadDim;  // 16 KB
constexpr int kMaxN = 256;
constexpr int kQTile = kMaxN * kHeadDim;  // 32 KB


struct __align__(1024) LgSmem {
  // n_st K-tile stages (two 64-token pages each, 128-byte swizzled rows) followed by the two
  // Q slots of NC * 128 bytes (the current and the next row block); see stage_count()
  uint8_t buf[kStages * kATile + 2 * kQTile];
  float sc[kStagesNarrow][2 * kPage];  // k_scale of the stage's two pages
  float w[kEpiWarps][kMaxN];       // head weights, one copy per epilogue warp
  int lens[kEpiWarps][8];          // row lengths of the current row block, per epilogue warp
  int hlen[kEpiWarps][8];          // histogram lengths of the current row block (0: no histogram)
  float* lrow[kEpiWarps][8];       // logits rows of the current row block
  uint32_t* mrow[kEpiWarps][8];    // mask rows (as 32-bit words) of the current row block
  int bq_ph[kProducers][2][32];    // producer batch (per producer warp): page ids of each item's two pages (-1: none)
  uint64_t full[kStagesNarrow];
  uint64_t empty[kStagesNarrow];   // 1 MMA commit + the 4 epilogue warps of the tile's team (they read sc[])
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

static_assert(kStagesNarrow * kATile + 2 * (kQTile / 2) <= kStages * kATile + 2 * kQTile, "stage layouts");

__host__ __device__ constexpr int stage_count(int nc) { return nc <= 128 ? kStagesNarrow : kStages; }

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
  const int32_t* hist_lens;  // fused pass-1 histogram: rows' histogram lengths, or null
  int32_t* zws;              // its workspace [ghist1 batch*4096 | ghist2 batch*4096 | cnt batch*2]
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

// Cursor over this CTA's contiguous range of (group, row block, tile) items,
// advanced without divisions.  init() positions it just before the first item.
struct Cursor {
  int g, sub, tile, len, tiles, n_sub, n_groups;
  __device__ void init(const PagedArgs& p, int g0, int l0) {
    g = g0;
    n_sub = (p.G + p.R - 1) / p.R;
    n_groups = p.batch / p.G;
    len = group_len(p, g);
    tiles = (len + kTileTok - 1) / kTileTok;
    sub = l0 / tiles;
    tile = l0 - sub * tiles - 1;
  }
  __device__ void next(const PagedArgs& p) {
    if (++tile >= tiles) {
      tile = 0;
      if (++sub >= n_sub) {
        sub = 0;
        do {
          if (++g >= n_groups) {  // never reached by callers that stay within their item count
            tiles = 1;
            break;
          }
          len = group_len(p, g);
          tiles = (len + kTileTok - 1) / kTileTok;
        } while (tiles == 0);
      }
    }
  }
};

// Index + phase parity of a ring of n slots (consumers wait on `phase`,
// producers of a "slot free" barrier wait on `phase ^ 1`).
struct Ring {
  int idx = 0, phase = 0;
  __device__ __forceinline__ void adv(int n) {
    if (++idx == n) {
      idx = 0;
      phase ^= 1;
    }
  }
};

// Fused pass 1 (mqa_hist.cu:219-226,239-272 of the reference): a token whose
// mask bit is set and that lies below the row's histogram length adds 1 to its
// key[31:20] bin and moves one count out of the +0 bin, where the init kernel
// put the whole length; positives are counted too.  One warp-row per call
// (every lane calls it).
__device__ __forceinline__ void pass1_count(const PagedArgs& p, int row, float s0, bool cnt) {
  int32_t* g1 = p.zws + static_cast<int64_t>(row) * kBins;
  const uint32_t key = to_key(s0);
  if (cnt) atomicAdd(g1 + (key >> 20), 1);
  const int nz = __popc(__ballot_sync(0xffffffffu, cnt));
  const int pos = __popc(__ballot_sync(0xffffffffu, cnt && key > kZeroKey));
  if ((threadIdx.x & 31) == 0 && nz) {
    int32_t* c = p.zws + 2 * static_cast<int64_t>(p.batch) * kBins + 2 * static_cast<int64_t>(row);
    atomicSub(g1 + kZeroBin, nz);
    atomicSub(c + 1, nz);
    if (pos) atomicAdd(c, pos);
  }
}

// kHist: the fused pass-1 histogram (p.zws set); a separate instance so the
// common path's epilogue is compiled without it.
template <int H, bool kHist>
__global__ __launch_bounds__(kLgThreads, 1) void mqa_logits_paged_kernel(const __grid_constant__ CUtensorMap tm_kv,
                                                                        const __grid_constant__ CUtensorMap tm_sc,
                                                                        const __grid_constant__ CUtensorMap tm_q,
                                                                        const PagedArgs p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  LgSmem& sm = smem_aligned_1024<LgSmem>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_groups = p.batch / p.G;
  const int n_sub = (p.G + p.R - 1) / p.R;
  const int NC = p.R * H;  // TMEM columns per accumulator buffer
  const int NACC = NC <= 128 ? 4 : 2;
  const int n_st = stage_count(NC);
  uint8_t* const a_base = sm.buf;
  uint8_t* const q_base = sm.buf + n_st * kATile;  // slot i at q_base + i * NC * 128 (1024-aligned)

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
  // Mask words past each row's processed tiles (the tiles write their own words): zeroed here,
  // rows strided over the grid, by every CTA (also those without tiles), instead of a memset.
  for (int row = blockIdx.x; row < p.batch; row += gridDim.x) {
    const int tiles = (group_len(p, row / p.G) + kTileTok - 1) / kTileTok;
    uint32_t* mw = reinterpret_cast<uint32_t*>(p.mask) + static_cast<int64_t>(row) * (p.width / 32);
    for (int wd = tiles * (kTileTok / 32) + static_cast<int>(threadIdx.x); wd < p.width / 32; wd += blockDim.x)
      mw[wd] = 0u;
  }
  __syncthreads();
  const int count = sm.count;
  if (count <= 0) return;  // uniform: before any barrier init or TMEM allocation

  uint32_t ncols = 32;
  while (ncols < static_cast<uint32_t>(NACC * NC)) ncols <<= 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < n_st; ++s) {
      mbar_init(&sm.full[s], 1);  // the item's producer: one expect_tx arrival
      mbar_init(&sm.empty[s], 1 + 4);  // MMA commit + the 4 warps of the tile's team
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.qfull[i], 1);
      mbar_init(&sm.qempty[i], 1);
    }
    for (int i = 0; i < kMaxAcc; ++i) {
      mbar_init(&sm.tfull[i], 1);
      mbar_init(&sm.tempty[i], 4);
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

  if (warp == 0 || warp >= kProducerB) {
    // ------------------------------------------------ TMA producers
    // Every mbarrier / TMA instruction of a lone issuing thread costs ~200
    // cycles (its warp shares a scheduler with epilogue warps), so the items
    // are dealt round robin to kProducers warps: producer k issues both pages
    // and both scale boxes of items k, k + kProducers, ...  Each warp first
    // resolves the page ids of its next 32 items in parallel (one lane per
    // item) into shared memory; lane 0 then waits for the item's stage and
    // issues its boxes.  Stage of item i: i % n_st, tracked incrementally.
    const int role = warp == 0 ? 0 : warp - kProducerB + 1;
    const uint64_t pol = l2_evict_first_policy();  // pages are read once; keep L2 for the logits
    Cursor cur;  // every lane keeps an identical copy, positioned before item `it0`
    cur.init(p, sm.start_group, sm.start_local);
    int issued = 0, last_it = -1, ok = 1;
    int st_s = role, st_ph = 0;  // stage and phase of this producer's next item (item i: i % n_st, (i / n_st) & 1)
    for (int it0 = 0; it0 < count && ok; it0 += 32 * kProducers) {
      {
        Cursor c = cur;
        const int my = it0 + role + lane * kProducers;  // this lane's item
        int ph0 = -1, ph1 = -1;
        if (my < count) {
          for (int k = 0; k <= role + lane * kProducers; ++k) c.next(p);
          const int n_pg = (c.len + kPage - 1) / kPage;
          const int32_t* bt = p.bt + static_cast<int64_t>(c.g) * p.G * p.bt_stride;
          if (2 * c.tile < n_pg) ph0 = __ldg(bt + 2 * c.tile);
          if (2 * c.tile + 1 < n_pg) ph1 = __ldg(bt + 2 * c.tile + 1);
        }
        __syncwarp();
        sm.bq_ph[role][0][lane] = ph0;
        sm.bq_ph[role][1][lane] = ph1;
        // advance every lane's copy to the end of this window (item it0 + 32 * kProducers - 1);
        // only needed when the window does not reach past the range
        if (it0 + 32 * kProducers < count) {
          for (int k = 0; k < kProducers - 1 - role; ++k) c.next(p);
          cur.g = __shfl_sync(0xffffffffu, c.g, 31);
          cur.sub = __shfl_sync(0xffffffffu, c.sub, 31);
          cur.tile = __shfl_sync(0xffffffffu, c.tile, 31);
          cur.len = __shfl_sync(0xffffffffu, c.len, 31);
          cur.tiles = __shfl_sync(0xffffffffu, c.tiles, 31);
        }
        __syncwarp();
      }
      if (lane == 0) {
        for (int j = 0; j < 32; ++j) {
          const int it = it0 + role + j * kProducers;
          if (it >= count) break;
          const int s = st_s;
          if (!mbar_wait(&sm.empty[s], st_ph ^ 1, abort, &g_hcu_status)) {
            ok = 0;
            break;
          }
          const int ph0 = sm.bq_ph[role][0][j];
          const int ph1 = sm.bq_ph[role][1][j];
          const uint32_t bytes = (ph0 >= 0 ? kPageFp8Bytes + kPage * 4 : 0) + (ph1 >= 0 ? kPageFp8Bytes + kPage * 4 : 0);
          if (bytes) {
            mbar_arrive_expect_tx(&sm.full[s], bytes);
            if (ph0 >= 0) {
              tma_load_3d_hint(a_base + s * kATile, &tm_kv, &sm.full[s], 0, 0, ph0, pol);
              tma_load_2d_hint(sm.sc[s], &tm_sc, &sm.full[s], 0, ph0, pol);
            }
            if (ph1 >= 0) {
              tma_load_3d_hint(a_base + s * kATile + kPageFp8Bytes, &tm_kv, &sm.full[s], 0, 0, ph1, pol);
              tma_load_2d_hint(sm.sc[s] + kPage, &tm_sc, &sm.full[s], 0, ph1, pol);
            }
          } else {
            mbar_arrive(&sm.full[s]);  // no page in this tile (cannot happen for in-range items)
          }
          ++issued;
          last_it = it;
          st_s += kProducers;
          if (st_s >= n_st) {
            st_s -= n_st;
            st_ph ^= 1;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (lane == 0) {
      // Drain: every copy issued must land before the CTA may exit.
      // Only items no later item shares a stage with: an older phase of a reused stage
      // has the same parity as the current one and would never read as complete.
      for (int k = 0; k < issued; ++k) {
        const int it = last_it - k * kProducers;
        if (it + n_st < count) break;
        mbar_wait_drain(&sm.full[it % n_st], (it / n_st) & 1, &g_hcu_status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (also loads Q)
    // Q of the j-th distinct (group, row block) key goes to slot j & 1; the next
    // key's Q is prefetched as soon as the current one is in use.
    if (elect_one()) {
      Cursor cur;
      cur.init(p, sm.start_group, sm.start_local);
      Ring st, acc;
      int qkey = -1, kq = -1, nq = 0;
      uint32_t idesc = 0;
      bool ok = true;
      auto issue_q = [&](int n, int qrow) -> bool {
        const int slot = n & 1;
        if (!mbar_wait(&sm.qempty[slot], ((n >> 1) & 1) ^ 1, abort, &g_hcu_status)) return false;
        mbar_arrive_expect_tx(&sm.qfull[slot], static_cast<uint32_t>(NC * kHeadDim));
        tma_load_2d(q_base + slot * NC * kHeadDim, &tm_q, &sm.qfull[slot], 0, qrow);
        nq = n + 1;
        return true;
      };
      for (int it = 0; it < count && ok; ++it) {
        cur.next(p);
        const int key = cur.g * n_sub + cur.sub;
        if (key != qkey) {
          if (kq >= 0) tc_commit(&sm.qempty[kq & 1]);  // the slot frees when the old key's MMAs finish
          ++kq;
          if (nq <= kq && !issue_q(kq, (cur.g * p.G + cur.sub * p.R) * H)) break;
          if (!mbar_wait(&sm.qfull[kq & 1], (kq >> 1) & 1, abort, &g_hcu_status)) break;
          qkey = key;
          const int nr = min(p.R, p.G - cur.sub * p.R);
          idesc = idesc_e4m3_f32(128, nr * H);
          if (count - 1 - it > cur.tiles - 1 - cur.tile) {  // another key follows in this CTA's range
            Cursor nx = cur;
            nx.tile = nx.tiles - 1;
            nx.next(p);
            if (!issue_q(kq + 1, (nx.g * p.G + nx.sub * p.R) * H)) break;
          }
        }
        if (!mbar_wait(&sm.full[st.idx], st.phase, abort, &g_hcu_status)) break;
        if (!mbar_wait(&sm.tempty[acc.idx], acc.phase ^ 1, abort, &g_hcu_status)) break;
        tc_fence_after();
        const uint64_t adesc = sw128_kmajor_desc(smem_u32(a_base + st.idx * kATile));
        const uint64_t bdesc = sw128_kmajor_desc(smem_u32(q_base + (kq & 1) * NC * kHeadDim));
        const uint32_t d = tmem + static_cast<uint32_t>(acc.idx * NC);
#pragma unroll
        for (int k = 0; k < kHeadDim / 32; ++k)
          mma_f8f6f4(d, adesc + 2 * k, bdesc + 2 * k, idesc, k > 0 ? 1u : 0u);
        tc_commit(&sm.empty[st.idx]);
        tc_commit(&sm.tfull[acc.idx]);
        st.adv(n_st);
        acc.adv(NACC);
      }
      // every Q copy issued must land before the CTA may exit
      for (int n = nq > 2 ? nq - 2 : 0; n < nq; ++n) mbar_wait_drain(&sm.qfull[n & 1], (n >> 1) & 1, &g_hcu_status);
      tc_commit(&sm.done);
      mbar_wait_drain(&sm.done, 0, &g_hcu_status);
    }
  } else if (warp >= 2 && warp < 2 + kEpiWarps) {
    // ------------------------------------------------ epilogue (warps 2..13)
    // kTeams teams of four warps (one warp per TMEM lane quadrant) take the tiles
    // round robin, so kTeams tiles' TMEM-load / math / store chains are in flight
    // at once; each warp computes every row of its team's tiles for its 32 tokens.
    const int ew = warp - 2;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int team = ew >> 2;
    // A team waits on the TMEM buffer of its item; parity waits stay unambiguous only while a
    // team cannot run a whole buffer ring ahead of the MMA, i.e. with at most NACC teams.
    const int n_teams = kTeams < NACC ? kTeams : NACC;
    int turn = 0;  // it % n_teams
    float* wsm = sm.w[ew];
    int* lsm = sm.lens[ew];
    Cursor cur;
    cur.init(p, sm.start_group, sm.start_local);
    Ring st, acc;
    int qkey = -1;
    int nr = 0;
    for (int it = 0; it < count; ++it) {
      cur.next(p);
      const int s = st.idx;
      const int a = acc.idx;
      const int aph = acc.phase;
      st.adv(n_st);
      acc.adv(NACC);
      const bool mine = turn == team;
      if (++turn == n_teams) turn = 0;
      if (!mine) continue;
      const int key = cur.g * n_sub + cur.sub;
      const int row0 = cur.g * p.G + cur.sub * p.R;
      if (key != qkey) {
        nr = min(p.R, p.G - cur.sub * p.R);
        __syncwarp();
        for (int i = lane; i < nr * H; i += 32)
          wsm[i] = __ldg(p.weights + static_cast<int64_t>(row0) * H + i) * kReluScale;  // pre-scaled for relu_fma2
        if (lane < nr) {
          lsm[lane] = clamp_len(__ldg(p.ctx_lens + row0 + lane), p.width);
          if constexpr (kHist) {
            const int hl = clamp_len(__ldg(p.hist_lens + row0 + lane), p.width);
            sm.hlen[ew][lane] = hl > kTopK ? hl : 0;  // rows of at most kTopK tokens need no histogram
          }
          sm.lrow[ew][lane] = p.logits + static_cast<int64_t>(row0 + lane) * p.width;
          sm.mrow[ew][lane] = reinterpret_cast<uint32_t*>(p.mask) + static_cast<int64_t>(row0 + lane) * (p.width / 32);
        }
        __syncwarp();
        qkey = key;
      }
      const int tok_in_tile = quad * 32 + lane;
      const int tok_base = cur.tile * kTileTok + quad * 32;
      const int token = tok_base + lane;
      if (!mbar_wait(&sm.tfull[a], aph, abort, &g_hcu_status)) break;
      tc_fence_after();
      const float ksc = sm.sc[s][tok_in_tile];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[s]);  // this warp is done with the stage's scales
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(a * NC);
      for (int r = 0; r < nr; ++r) {
        // 8 independent chains: 4 packed fp32 pairs
        float2 acc0 = make_float2(0.f, 0.f), acc1 = acc0, acc2 = acc0, acc3 = acc0;
        if constexpr (kPgChunked) {
#pragma unroll
          for (int c = 0; c < H / 32; ++c) {
            uint32_t v[32];
            tmem_ld_x32_sync(tbase + r * H + c * 32, v);
            const float4* w4 = reinterpret_cast<const float4*>(wsm + r * H + c * 32);
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              const float4 wa = w4[j];
              const float4 wb = w4[j + 1];
              const uint32_t* x = &v[4 * j];
              relu_fma2(acc0, x[0], x[1], wa.x, wa.y);
              relu_fma2(acc1, x[2], x[3], wa.z, wa.w);
              relu_fma2(acc2, x[4], x[5], wb.x, wb.y);
              relu_fma2(acc3, x[6], x[7], wb.z, wb.w);
            }
          }
        } else {
          uint32_t v[H / 32][32];
#pragma unroll
          for (int c = 0; c < H / 32; ++c) tmem_ld_x32(tbase + r * H + c * 32, v[c]);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < H / 32; ++c) tmem_reg_fence(v[c]);
#pragma unroll
          for (int c = 0; c < H / 32; ++c) {
            const float4* w4 = reinterpret_cast<const float4*>(wsm + r * H + c * 32);
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              const float4 wa = w4[j];
              const float4 wb = w4[j + 1];
              const uint32_t* x = &v[c][4 * j];
              relu_fma2(acc0, x[0], x[1], wa.x, wa.y);
              relu_fma2(acc1, x[2], x[3], wa.z, wa.w);
              relu_fma2(acc2, x[4], x[5], wb.x, wb.y);
              relu_fma2(acc3, x[6], x[7], wb.z, wb.w);
            }
          }
        }
        float s0 = ((acc0.x + acc0.y) + (acc1.x + acc1.y)) + ((acc2.x + acc2.y) + (acc3.x + acc3.y));
        s0 *= ksc;
        const bool keep = token < lsm[r] && __float_as_uint(s0) != 0u;
        const uint32_t bits = __ballot_sync(0xffffffffu, keep);
        st_u32_if(sm.mrow[ew][r] + (tok_base >> 5), bits, lane == 0 && tok_base < p.width);
        st_f32_if(sm.lrow[ew][r] + token, s0, keep);
        if constexpr (kHist) {
          const int hl = sm.hlen[ew][r];
          if (hl) pass1_count(p, row0 + r, s0, keep && token < hl);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.tempty[a]);
    }
  }

  // Programmatic dependent launch: the next kernel of the stream (the top-k) may be scheduled once
  // every CTA got here; it still waits (griddepcontrol.wait) for this grid's completion and writes.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

// ---------------------------------------------------------------- ragged (prefill) kernel
//
// mqa_logits_ragged_kernel: query row r sees tokens [rs[r], re[r]) of a
// contiguous fp8 K.  Rows are grouped into super-blocks of kQB row blocks of
// RB = 256 / H rows (16 rows at H = 64); a CTA keeps one super-block's Q (4 x
// 32 KB) resident and streams the 128-token K tiles the super-block sees
// through a 4-stage TMA ring.  Each K tile feeds kQB MMAs (M = 128 tokens,
// N = 256 query heads) into two 256-column TMEM accumulators, i.e. 2 KFLOP per
// K byte.  The work list is (super-block, tile), cut into one contiguous range
// per CTA on the device.  Same logits / mask contract as the paged kernel.
constexpr int kPfStages = 4;
constexpr int kQB = 4;
constexpr int kPfEpiWarps = 16;  // warps 2..17: kPfTeams per TMEM lane quadrant
constexpr int kPfTeams = kPfEpiWarps / 4;  // warp t of a quadrant takes rows r % kPfTeams == t of every row block
constexpr int kPfThreads = (2 + kPfEpiWarps) * 32;

struct __align__(1024) PfSmem {
  uint8_t q[kQB][kQTile];
  uint8_t a[kPfStages][kATile];
  float w[kPfEpiWarps][kQB * kMaxN / kPfTeams];  // weights of the rows this epilogue warp owns
  int rs[kPfEpiWarps][16];          // first visible token of each owned row
  int re[kPfEpiWarps][16];          // visible length of each owned row
  float* lrow[kPfEpiWarps][16];     // logits row of each owned row (super-block); kCand: its list
  uint32_t* mrow[kPfEpiWarps][16];  // mask row (as 32-bit words) of each owned row; kCand: its count
  uint32_t lo[kPfEpiWarps][16];     // kCand: the owned rows' bounds as keys
  int2 cfifo[kPfEpiWarps][2][32];  // kCand: each warp's two staging halves
  uint64_t full[kPfStages];
  uint64_t empty[kPfStages];
  uint64_t qfull;
  uint64_t qempty;
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t done;
  uint32_t tmem_base;
  int start_sb;
  int start_local;
  int count;
  int abort;
};

struct RaggedArgs {
  const float* k_scale;
  const float* weights;
  const int32_t* rs;
  const int32_t* re;
  float* logits;
  int16_t* mask;
  int64_t stride;  // logits row stride (elements), multiple of 64
  int rows;
  int n_tokens;
  // kCand (the fused prefill top-k): instead of logits and mask, every visible token whose key is
  // at or above the row's bound is appended as (key, token) to the row's list cand[row * cand_cap ..]
  // (cand_cnt[row] counts all of them, also past cand_cap); rows of at most cand_all_len visible
  // tokens take every visible token.
  const int32_t* bounds;  // order-preserving int32 (key ^ 0x80000000)
  int32_t* cand_cnt;
  int2* cand;
  int cand_cap;
  int cand_all_len;
  const int32_t* run_if;  // non-null: the launch does nothing while *run_if == 0
};

// kCand staging: each epilogue warp collects its candidates (key, token | owned-row slot << 24) in
// one of two 32-entry shared-memory halves.  When a warp-row's entries do not fit the current half,
// the warp seals it -- one slot-reservation atomic per owned row with entries, issued together and
// not waited for -- and switches halves; the sealed half's entries are written to the rows' global
// lists at the next seal (or before the owned rows change), when the reservations have long
// arrived.  So no epilogue warp waits on a global atomic in the steady state.
struct CandStage {
  int fill = 0;      // entries in the current half
  int half = 0;      // the current half
  int pend = 0;      // entries of the sealed half (0: none pending)
  int base = 0;      // lane s < NS: the sealed half's first slot in owned row s
};

// Per-slot ballots of a half's entries: lane i holds entry i (slot sl, -1 past `fill`).
template <int NS>
__device__ __forceinline__ void cand_slots(const int2* half, int fill, int lane, int2& e, int& sl, int& pre, int& n_s) {
  e = lane < fill ? half[lane] : make_int2(0, 0);
  sl = lane < fill ? (e.y >> 24) : -1;
  pre = 0;
  n_s = 0;
#pragma unroll
  for (int q = 0; q < NS; ++q) {
    const uint32_t m = __ballot_sync(0xffffffffu, sl == q);
    if (sl == q) pre = __popc(m & ((1u << lane) - 1u));
    if (lane == q) n_s = __popc(m);
  }
}

// Seal: reserve list slots for the current half (the returned base is consumed by cand_complete).
template <int NS>
__device__ __forceinline__ int cand_seal(const int2* half, int fill, uint32_t* const* mrow, int lane) {
  int2 e;
  int sl, pre, n_s;
  cand_slots<NS>(half, fill, lane, e, sl, pre, n_s);
  return (lane < NS && n_s > 0) ? atomicAdd(reinterpret_cast<int*>(mrow[lane]), n_s) : 0;
}

// Complete: write a sealed half's entries at their reserved slots.
template <int NS>
__device__ __forceinline__ void cand_complete(const int2* half, int fill, int base, float* const* lrow, int cap,
                                              int lane) {
  int2 e;
  int sl, pre, n_s;
  cand_slots<NS>(half, fill, lane, e, sl, pre, n_s);
  const int b = __shfl_sync(0xffffffffu, base, sl < 0 ? 0 : sl);
  if (sl >= 0 && b + pre < cap) reinterpret_cast<int2*>(lrow[sl])[b + pre] = make_int2(e.x, e.y & 0xFFFFFF);
}

// Appends this warp-row's candidates (lanes with c; bal = their ballot), sealing first when they
// do not fit the current half.
template <int NS>
__device__ __forceinline__ void cand_append(CandStage& st, int2 (*halves)[32], float* const* lrow,
                                            uint32_t* const* mrow, int cap, int lane, bool c, uint32_t bal, int2 ent) {
  const int k = __popc(bal);
  if (st.fill + k > 32) {
    __syncwarp();  // the current half's entries are visible to every lane
    if (st.pend) cand_complete<NS>(halves[st.half ^ 1], st.pend, st.base, lrow, cap, lane);
    st.base = cand_seal<NS>(halves[st.half], st.fill, mrow, lane);
    st.pend = st.fill;
    st.half ^= 1;
    st.fill = 0;
    __syncwarp();  // the completed half is free
  }
  if (c) halves[st.half][st.fill + __popc(bal & ((1u << lane) - 1u))] = ent;
  st.fill += k;
}

// Writes out everything staged (before the owned rows change, and at the end).
template <int NS>
__device__ __forceinline__ void cand_drain(CandStage& st, int2 (*halves)[32], float* const* lrow,
                                           uint32_t* const* mrow, int cap, int lane) {
  __syncwarp();
  if (st.pend) cand_complete<NS>(halves[st.half ^ 1], st.pend, st.base, lrow, cap, lane);
  if (st.fill) {
    const int base = cand_seal<NS>(halves[st.half], st.fill, mrow, lane);
    cand_complete<NS>(halves[st.half], st.fill, base, lrow, cap, lane);
  }
  st.pend = 0;
  st.fill = 0;
  __syncwarp();
}

template <int H>
__device__ __forceinline__ void sb_tiles(const RaggedArgs& p, int sb, int& t0, int& tiles) {
  constexpr int RB = kMaxN / H;
  constexpr int SBR = kQB * RB;
  int lo = INT32_MAX, hi = 0;
  const int r1 = min(p.rows, (sb + 1) * SBR);
  for (int r = sb * SBR; r < r1; ++r) {
    const int a = max(__ldg(p.rs + r), 0);
    const int e = min(__ldg(p.re + r), p.n_tokens);
    if (e > a) {
      lo = min(lo, a);
      hi = max(hi, e);
    }
  }
  if (hi <= lo) {
    t0 = 0;
    tiles = 0;
  } else {
    t0 = lo / kTileTok;
    tiles = (hi + kTileTok - 1) / kTileTok - t0;
  }
}

template <int H>
struct RCursor {
  int sb, li, t0, tiles;
  __device__ void init(const RaggedArgs& p, int sb0, int l0) {
    sb = sb0;
    li = l0;
    sb_tiles<H>(p, sb, t0, tiles);
  }
  __device__ int next(const RaggedArgs& p) {  // returns the absolute tile index
    while (li >= tiles) {
      ++sb;
      li = 0;
      sb_tiles<H>(p, sb, t0, tiles);
    }
    return t0 + li++;
  }
};

template <int H, bool kMixed, bool kCand>
__global__ __launch_bounds__(kPfThreads, 1) void mqa_logits_ragged_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                                         const __grid_constant__ CUtensorMap tm_q,
                                                                         const RaggedArgs p) {
  constexpr int RB = kMaxN / H;  // rows per row block (N = 256)
  constexpr int SBR = kQB * RB;  // rows per super-block
  if (p.run_if != nullptr && __ldcg(p.run_if) == 0) return;  // grid-uniform, before any barrier or TMEM use
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  PfSmem& sm = smem_aligned_1024<PfSmem>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_sb = (p.rows + SBR - 1) / SBR;

  if (warp == 0) {
    int64_t total = 0;
    for (int base = 0; base < n_sb; base += 32) {
      int t0, c = 0;
      if (base + lane < n_sb) sb_tiles<H>(p, base + lane, t0, c);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
      total += c;
    }
    const int64_t begin = total * blockIdx.x / gridDim.x;
    const int64_t end = total * (blockIdx.x + 1) / gridDim.x;
    int sg = 0, sl = 0;
    if (end > begin) {
      int64_t run = 0;
      for (int base = 0; base < n_sb; base += 32) {
        int t0, c = 0;
        if (base + lane < n_sb) sb_tiles<H>(p, base + lane, t0, c);
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
      sm.start_sb = sg;
      sm.start_local = sl;
      sm.count = static_cast<int>(end - begin);
    }
  }
  __syncthreads();
  const int count = sm.count;
  if (count <= 0) return;

  constexpr uint32_t ncols = 512;  // two 256-column accumulators
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);  // the MMAs are the stage's only reader
    }
    mbar_init(&sm.qfull, 1);
    mbar_init(&sm.qempty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.tfull[i], 1);
      mbar_init(&sm.tempty[i], kPfEpiWarps);
    }
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_k);
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
    // ------------------------------------------------ TMA producer
    if (elect_one()) {
      RCursor<H> cur;
      cur.init(p, sm.start_sb, sm.start_local);
      int qsb = -1, qn = 0, issued = 0;
      for (int it = 0; it < count; ++it) {
        const int tile = cur.next(p);
        if (cur.sb != qsb) {
          if (!mbar_wait(&sm.qempty, (qn & 1) ^ 1, abort, &g_hcu_status)) break;
          const int row0 = cur.sb * SBR;
          const int nrb = min(kQB, (p.rows - row0 + RB - 1) / RB);
          mbar_arrive_expect_tx(&sm.qfull, static_cast<uint32_t>(nrb * kQTile));
          for (int j = 0; j < nrb; ++j) tma_load_2d(sm.q[j], &tm_q, &sm.qfull, 0, (row0 + j * RB) * H);
          ++qn;
          qsb = cur.sb;
        }
        const int s = it % kPfStages;
        if (!mbar_wait(&sm.empty[s], ((it / kPfStages) & 1) ^ 1, abort, &g_hcu_status)) break;
        mbar_arrive_expect_tx(&sm.full[s], static_cast<uint32_t>(kATile));
        tma_load_2d(sm.a[s], &tm_k, &sm.full[s], 0, tile * kTileTok);
        issued = it + 1;
      }
      const int first = issued > kPfStages ? issued - kPfStages : 0;
      for (int it = first; it < issued; ++it)
        mbar_wait_drain(&sm.full[it % kPfStages], (it / kPfStages) & 1, &g_hcu_status);
      if (qn > 0) mbar_wait_drain(&sm.qfull, (qn - 1) & 1, &g_hcu_status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (elect_one()) {
      RCursor<H> cur;
      cur.init(p, sm.start_sb, sm.start_local);
      int qsb = -1, qn = 0, nrb = 0, u = 0;
      bool ok = true;
      for (int it = 0; it < count && ok; ++it) {
        cur.next(p);
        if (cur.sb != qsb) {
          if (qn > 0) tc_commit(&sm.qempty);
          if (!mbar_wait(&sm.qfull, qn & 1, abort, &g_hcu_status)) break;
          ++qn;
          qsb = cur.sb;
          nrb = min(kQB, (p.rows - cur.sb * SBR + RB - 1) / RB);
        }
        const int s = it % kPfStages;
        if (!mbar_wait(&sm.full[s], (it / kPfStages) & 1, abort, &g_hcu_status)) break;
        const uint64_t adesc = sw128_kmajor_desc(smem_u32(sm.a[s]));
        for (int j = 0; j < nrb; ++j, ++u) {
          const int a = u & 1;
          if (!mbar_wait(&sm.tempty[a], ((u >> 1) & 1) ^ 1, abort, &g_hcu_status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nr = min(RB, p.rows - (cur.sb * SBR + j * RB));
          const uint32_t idesc = idesc_e4m3_f32(128, nr * H);
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sm.q[j]));
          const uint32_t d = tmem + static_cast<uint32_t>(a * kMaxN);
#pragma unroll
          for (int k = 0; k < kHeadDim / 32; ++k)
            mma_f8f6f4(d, adesc + 2 * k, bdesc + 2 * k, idesc, k > 0 ? 1u : 0u);
          tc_commit(&sm.tfull[a]);
        }
        if (ok) tc_commit(&sm.empty[s]);
      }
      tc_commit(&sm.done);
      mbar_wait_drain(&sm.done, 0, &g_hcu_status);
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..17)
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int rsel = ew >> 2;  // rows r % kPfTeams == rsel of every row block
    constexpr int RPW = RB / kPfTeams;  // rows per row block owned by this warp
    float* wsm = sm.w[ew];
    int* rs = sm.rs[ew];
    int* re = sm.re[ew];
    RCursor<H> cur;
    cur.init(p, sm.start_sb, sm.start_local);
    int qsb = -1, nrb = 0, u = 0;
    bool ok = true;
    CandStage cst;  // kCand: this warp's staged candidates
    for (int it = 0; it < count && ok; ++it) {
      const int tile = cur.next(p);
      const int row0 = cur.sb * SBR;
      if (cur.sb != qsb) {
        qsb = cur.sb;
        nrb = min(kQB, (p.rows - row0 + RB - 1) / RB);
        if constexpr (kCand) {  // before the owned rows change
          cand_drain<kQB * RPW>(cst, sm.cfifo[ew], sm.lrow[ew], sm.mrow[ew], p.cand_cap, lane);
        }
        __syncwarp();
        for (int lr = 0; lr < kQB * RPW; ++lr) {
          const int row = row0 + (lr / RPW) * RB + (lr % RPW) * kPfTeams + rsel;
          const bool in = row < p.rows;
          for (int h = lane; h < H; h += 32)  // pre-scaled by 2^25 where the ReLU is the saturating FMA
            wsm[lr * H + h] = in ? __ldg(p.weights + static_cast<int64_t>(row) * H + h) *
                                       ((kMixed && (h & 1)) ? 1.f : kReluScale)
                                 : 0.f;
          if (lane == 0) {
            const int a0 = in ? max(__ldg(p.rs + row), 0) : 0;
            const int e0 = in ? min(__ldg(p.re + row), p.n_tokens) : 0;
            rs[lr] = a0;
            re[lr] = e0 > a0 ? e0 - a0 : 0;  // visible length: token is visible iff (unsigned)(token - rs) < len
            if constexpr (kCand) {
              // the row's list and count in place of its logits and mask rows; its bound as a key
              const int64_t r = in ? row : 0;
              sm.lrow[ew][lr] = reinterpret_cast<float*>(p.cand + r * p.cand_cap);
              sm.mrow[ew][lr] = reinterpret_cast<uint32_t*>(p.cand_cnt + r);
              sm.lo[ew][lr] = !in ? 0xFFFFFFFFu
                                  : (re[lr] <= p.cand_all_len ? 0u : static_cast<uint32_t>(__ldg(p.bounds + row)) ^ kZeroKey);
            } else {
              sm.lrow[ew][lr] = p.logits + static_cast<int64_t>(in ? row : 0) * p.stride;
              sm.mrow[ew][lr] = reinterpret_cast<uint32_t*>(p.mask) + static_cast<int64_t>(in ? row : 0) * (p.stride / 32);
            }
          }
        }
        __syncwarp();
      }
      const int tok_base = tile * kTileTok + quad * 32;
      const int token = tok_base + lane;
      // k_scale of this thread's token: contiguous K, so a plain load issued before the wait
      const float ksc = token < p.n_tokens ? __ldg(p.k_scale + token) : 0.f;
      const bool mstore = lane == 0 && tok_base < p.stride;  // this warp's 32-bit mask word exists
      const int mword = tok_base >> 5;
      for (int j = 0; j < nrb; ++j, ++u) {
        const int a = u & 1;
        if (!mbar_wait(&sm.tfull[a], (u >> 1) & 1, abort, &g_hcu_status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(a * kMaxN);
        const int nr = min(RB, p.rows - (row0 + j * RB));
        for (int r = rsel, lr = j * RPW; r < nr; r += kPfTeams, ++lr) {
          // one 32-head TMEM chunk at a time keeps the epilogue within the 18-warp register budget
          float2 acc0 = make_float2(0.f, 0.f), acc1 = acc0, acc2 = acc0, acc3 = acc0;
#pragma unroll
          for (int c = 0; c < H / 32; ++c) {
            uint32_t v[32];
            tmem_ld_x32(tbase + r * H + c * 32, v);
            tmem_ld_wait();
            tmem_reg_fence(v);
            const float4* w4 = reinterpret_cast<const float4*>(wsm + lr * H + c * 32);
#pragma unroll
            for (int jj = 0; jj < 8; jj += 2) {
              const float4 wa = w4[jj];
              const float4 wb = w4[jj + 1];
              const uint32_t* x = &v[4 * jj];
              if constexpr (kMixed) {
                relu_fma2_mixed(acc0, x[0], x[1], wa.x, wa.y);
                relu_fma2_mixed(acc1, x[2], x[3], wa.z, wa.w);
                relu_fma2_mixed(acc2, x[4], x[5], wb.x, wb.y);
                relu_fma2_mixed(acc3, x[6], x[7], wb.z, wb.w);
              } else {
                relu_fma2_pk(acc0, x[0], x[1], make_float2(wa.x, wa.y));
                relu_fma2_pk(acc1, x[2], x[3], make_float2(wa.z, wa.w));
                relu_fma2_pk(acc2, x[4], x[5], make_float2(wb.x, wb.y));
                relu_fma2_pk(acc3, x[6], x[7], make_float2(wb.z, wb.w));
              }
            }
          }
          float s0 = ((acc0.x + acc0.y) + (acc1.x + acc1.y)) + ((acc2.x + acc2.y) + (acc3.x + acc3.y));
          s0 *= ksc;
          if constexpr (kCand) {
            // key of a visible token: to_key(+0) is the +0 key an unset mask bit stands for, so the
            // keys equal those the top-k derives from the logits and mask
            const uint32_t key = to_key(s0);
            const bool c = static_cast<uint32_t>(token - rs[lr]) < static_cast<uint32_t>(re[lr]) && key >= sm.lo[ew][lr];
            const uint32_t bal = __ballot_sync(0xffffffffu, c);
            cand_append<kQB * RPW>(cst, sm.cfifo[ew], sm.lrow[ew], sm.mrow[ew], p.cand_cap, lane, c, bal,
                                   make_int2(static_cast<int>(key), token | (lr << 24)));
          } else {
            const bool keep = static_cast<uint32_t>(token - rs[lr]) < static_cast<uint32_t>(re[lr]) &&
                              __float_as_uint(s0) != 0u;
            const uint32_t bits = __ballot_sync(0xffffffffu, keep);
            st_u32_if(sm.mrow[ew][lr] + mword, bits, mstore);
            st_f32_if(sm.lrow[ew][lr] + token, s0, keep);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.tempty[a]);
      }
    }
    if constexpr (kCand) cand_drain<kQB * RPW>(cst, sm.cfifo[ew], sm.lrow[ew], sm.mrow[ew], p.cand_cap, lane);
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

int map_error(const char* what) {
  set_last_error_msg("cuTensorMapEncodeTiled rejected the tensor map of ", what);
  return HCU_ERR_LAUNCH;
}

template <int H, bool kHist>
int launch_paged_t(const CUtensorMap& tkv, const CUtensorMap& tsc, const CUtensorMap& tq, const PagedArgs& a,
                   cudaStream_t stream) {
  const size_t smem = sizeof(LgSmem) + 1024;
  cudaFuncSetAttribute(mqa_logits_paged_kernel<H, kHist>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  mqa_logits_paged_kernel<H, kHist><<<sm_count(), kLgThreads, smem, stream>>>(tkv, tsc, tq, a);
  return launch_status();
}

template <int H, bool kMixed, bool kCand = false>
void launch_ragged(const CUtensorMap& tk, const CUtensorMap& tq, const RaggedArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(PfSmem) + 1024;
  cudaFuncSetAttribute(mqa_logits_ragged_kernel<H, kMixed, kCand>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  mqa_logits_ragged_kernel<H, kMixed, kCand><<<sm_count(), kPfThreads, smem, st>>>(tk, tq, a);
}

template <int H>
int launch_paged(const CUtensorMap& tkv, const CUtensorMap& tsc, const CUtensorMap& tq, const PagedArgs& a,
                 cudaStream_t stream) {
  return a.zws ? launch_paged_t<H, true>(tkv, tsc, tq, a, stream) : launch_paged_t<H, false>(tkv, tsc, tq, a, stream);
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
  CUtensorMap tkv, tsc, tq;
  if (!make_map_pages(&tkv, kv_cache, static_cast<uint64_t>(n_pages), static_cast<uint64_t>(page_stride)))
    return map_error("kv_cache pages");
  if (!make_map_page_scales(&tsc, kv_cache, static_cast<uint64_t>(n_pages), static_cast<uint64_t>(page_stride)))
    return map_error("kv_cache scales");
  if (!make_map_2d(&tq, q, kHeadDim, static_cast<uint64_t>(batch * heads), kHeadDim, kHeadDim,
                   static_cast<uint32_t>(R * heads), CU_TENSOR_MAP_SWIZZLE_128B))
    return map_error("q");
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
  a.hist_lens = hist_lens;
  a.zws = hist_lens ? zws : nullptr;
  a.batch = static_cast<int>(batch);
  a.G = static_cast<int>(group_size);
  a.R = static_cast<int>(R);
  a.width = static_cast<int>(max_context_len);
  if (hist_lens) {  // the workspace's bins and counts, filled by the kernel's epilogue
    const int hs = launch_hist_init(zws, hist_lens, batch, max_context_len, st);
    if (hs != HCU_OK) return hs;
  }
  return heads == 64 ? launch_paged<64>(tkv, tsc, tq, a, st) : launch_paged<32>(tkv, tsc, tq, a, st);
}

namespace hcu {
// Ragged logits launch without the mask memset (internal: the fused prefill top-k).  Rows see
// [row_start, row_end); with bounds set, the candidate-list epilogue replaces the logits and mask
// stores (logits and mask may then be null); run_if predicates the launch on a device word.
int launch_ragged_logits(const uint8_t* q, int64_t rows, int64_t heads, const uint8_t* k_fp8, const float* k_scale,
                         int64_t n_tokens, const float* weights, const int32_t* row_start, const int32_t* row_end,
                         float* logits, int64_t logits_stride, int16_t* mask, const int32_t* bounds,
                         int32_t* cand_cnt, int2* cand, int cand_cap, int cand_all_len, const int32_t* run_if,
                         cudaStream_t st) {
  if (rows == 0 || n_tokens == 0) return HCU_OK;
  CUtensorMap tk, tq;
  const int RB = static_cast<int>(kMaxN / heads);
  if (!make_map_2d(&tk, k_fp8, kHeadDim, static_cast<uint64_t>(n_tokens), kHeadDim, kHeadDim, kTileTok,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return map_error("k_fp8");
  if (!make_map_2d(&tq, q, kHeadDim, static_cast<uint64_t>(rows * heads), kHeadDim, kHeadDim,
                   static_cast<uint32_t>(RB * heads), CU_TENSOR_MAP_SWIZZLE_128B))
    return map_error("q");
  RaggedArgs a{};
  a.k_scale = k_scale;
  a.weights = weights;
  a.rs = row_start;
  a.re = row_end;
  a.logits = logits;
  a.mask = mask;
  a.stride = logits_stride;
  a.rows = static_cast<int>(rows);
  a.n_tokens = static_cast<int>(n_tokens);
  a.bounds = bounds;
  a.cand_cnt = cand_cnt;
  a.cand = cand;
  a.cand_cap = cand_cap;
  a.cand_all_len = cand_all_len;
  a.run_if = run_if;
  static const bool mixed = [] {
    const char* e = std::getenv("HCU_PF_RELU");
    return e != nullptr && e[0] == 'm';
  }();
  if (bounds != nullptr) {
    if (heads == 64)
      launch_ragged<64, false, true>(tk, tq, a, st);
    else
      launch_ragged<32, false, true>(tk, tq, a, st);
  } else if (heads == 64) {
    mixed ? launch_ragged<64, true>(tk, tq, a, st) : launch_ragged<64, false>(tk, tq, a, st);
  } else {
    mixed ? launch_ragged<32, true>(tk, tq, a, st) : launch_ragged<32, false>(tk, tq, a, st);
  }
  return launch_status();
}
}  // namespace hcu

extern "C" int hcu_mqa_logits_ragged(const uint8_t* q, int64_t rows, int64_t heads, const uint8_t* k_fp8,
                                     const float* k_scale, int64_t n_tokens, const float* weights,
                                     const int32_t* row_start, const int32_t* row_end, float* logits,
                                     int64_t logits_stride, int16_t* mask, hcu_stream_t stream) {
  using namespace hcu;
  if (heads != 32 && heads != 64) return HCU_ERR_UNSUPPORTED;
  if (rows < 0 || n_tokens < 0 || rows * heads > INT32_MAX || n_tokens > INT32_MAX) return HCU_ERR_ARG;
  if (logits_stride < n_tokens || logits_stride % 64 != 0) return HCU_ERR_ARG;
  if (rows == 0) return HCU_OK;
  if (!q || !k_fp8 || !k_scale || !weights || !row_start || !row_end || !logits || !mask) return HCU_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_fp8) | reinterpret_cast<uintptr_t>(k_scale) |
       reinterpret_cast<uintptr_t>(mask) | reinterpret_cast<uintptr_t>(weights)) % 16 != 0)
    return HCU_ERR_ARG;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(mask, 0, static_cast<size_t>(rows * (logits_stride / 16)) * sizeof(int16_t), st) != cudaSuccess)
    return launch_status();
  return launch_ragged_logits(q, rows, heads, k_fp8, k_scale, n_tokens, weights, row_start, row_end, logits,
                              logits_stride, mask, nullptr, nullptr, nullptr, 0, 0, nullptr, st);
}
