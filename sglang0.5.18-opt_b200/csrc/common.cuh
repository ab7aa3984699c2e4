// Shared device helpers for the sm_100a indexer kernels: status word, bounded
// mbarrier waits, TMA and tcgen05 wrappers (inline PTX), key transform.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hcu_indexer.h"

namespace hcu {

constexpr int kTopK = 2048;
constexpr int kPage = 64;
constexpr int kHeadDim = 128;
constexpr int kPageFp8Bytes = kPage * kHeadDim;  // 8192
constexpr uint32_t kZeroKey = 0x80000000u;
constexpr int kBins = 4096;
constexpr int kZeroBin = 0x800;

// A bounded wait gives up after g_hcu_wait_limit_ns nanoseconds of %globaltimer
// (default kWaitLimitNs; hcu_set_wait_limit_ns changes it).  Every legitimate
// wait in these kernels is microseconds to milliseconds long.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Monotone float -> uint32 key: larger float <=> larger key; -0 < +0.
// (Same transform as hcu_ops/csrc/sparse_mask_topk.cu:40-43 of the reference.)
__device__ __forceinline__ uint32_t to_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

}  // namespace hcu

// Per-translation-unit wait limit (no relocatable device code: each unit that
// waits keeps its own copy, set through its hcu::set_wait_limit_* accessor).
static __device__ uint64_t g_hcu_wait_limit_ns = hcu::kWaitLimitNs;

namespace hcu {

__device__ __forceinline__ uint64_t wait_limit_ns() {
  return *reinterpret_cast<volatile uint64_t*>(&g_hcu_wait_limit_ns);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Suspend-time hint of a waiting thread (ns): the hardware parks the warp until
// the phase completes or the hint elapses, so waiting warps do not spin on the
// issue slots that the working warps of the same SM sub-partition need.
constexpr uint32_t kSuspendHintNs = 200000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Gives up after the
// wait limit (or at once when *abort is set by another warp), records
// HCU_STATUS_WAIT_TIMEOUT in `status`, sets *abort and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          unsigned int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  const uint64_t lim = wait_limit_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > lim) {
      atomicOr(status, HCU_STATUS_WAIT_TIMEOUT);
      *abort = 1;
      return false;
    }
  }
}

// Same wait without the abort short-cut: used to drain copies already issued.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, unsigned int* status) {
  const uint64_t t0 = globaltimer();
  const uint64_t lim = wait_limit_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > lim) {
      atomicOr(status, HCU_STATUS_WAIT_TIMEOUT);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------- cross-GPU flags
// System-scope release store / acquire load of a 32-bit flag (another GPU
// writes or reads it over NVLink).
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// L2 policy for data read exactly once (streamed K-cache pages): evicted first,
// so it does not push out data a later kernel re-reads (the logits just written).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_1d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0) {
  asm volatile(
      "cp.async.bulk.tensor.1d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0)
      : "memory");
}

// Packed fp32 pair FMA (sm_100): d = a * b + c elementwise on two lanes of a 64-bit register.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
        "l"(*reinterpret_cast<uint64_t*>(&c)));
  return *reinterpret_cast<float2*>(&d);
}

// Scale of the saturating ReLU below: 2^25 exceeds |q . k| for any fp8 e4m3
// q, k of 128 dims (128 * 448 * 448 < 2^25), so sat(x * 2^-25) = relu(x) * 2^-25
// exactly (power-of-two scaling, clamped to [0, 1], NaN -> 0).
constexpr float kReluScale = 33554432.f;  // 2^25

// acc += relu(x) * w on a pair of lanes, where w2 = w * 2^25 (the caller
// pre-scales the weights): the ReLU is one saturating fma.rn.sat.f32 per lane
// on the FMA pipe and the two products go through one fma.rn.f32x2.  The
// result equals fma(relu(x), w, acc) bit for bit (both scalings are exact;
// weights must satisfy |w| < 2^102, where w * relu(x) itself nears overflow).
__device__ __forceinline__ void relu_fma2(float2& acc, uint32_t x0, uint32_t x1, float w0, float w1) {
  asm("{\n\t"
      ".reg .f32 a, b;\n\t"
      ".reg .b64 p, q, r;\n\t"
      "fma.rn.sat.f32 a, %2, 0f33000000, 0f00000000;\n\t"
      "fma.rn.sat.f32 b, %3, 0f33000000, 0f00000000;\n\t"
      "mov.b64 p, {a, b};\n\t"
      "mov.b64 q, {%4, %5};\n\t"
      "mov.b64 r, {%0, %1};\n\t"
      "fma.rn.f32x2 r, p, q, r;\n\t"
      "mov.b64 {%0, %1}, r;\n\t"
      "}"
      : "+f"(acc.x), "+f"(acc.y)
      : "f"(__uint_as_float(x0)), "f"(__uint_as_float(x1)), "f"(w0), "f"(w1));
}

// The same step with the compiler's packed-FMA intrinsic: relu(x) * 2^-25 as a
// saturating multiply (exact scaling; the saturation clamps negatives, -0 and
// NaN to +0 and never reaches 1 since |x| < 2^25), then one fma.rn.f32x2 with
// the pre-scaled weight pair.  Bit-identical to relu_fma2; the register pairs are
// left to the compiler.
__device__ __forceinline__ void relu_fma2_pk(float2& acc, uint32_t x0, uint32_t x1, float2 w) {
  const float2 r = make_float2(__saturatef(__uint_as_float(x0) * 0x1p-25f), __saturatef(__uint_as_float(x1) * 0x1p-25f));
  acc = __ffma2_rn(r, w, acc);
}

// The same sum with the ReLU split over two pipes: lane x0 through the
// saturating FMA (its weight w0 pre-scaled by 2^25), lane x1 through max.f32 on
// the ALU pipe (w1 unscaled; max returns 0 for a NaN x1, like fmaxf).  Both
// products are exact scalings of relu(x) * w, so the result equals
// relu_fma2's bit for bit while the FMA pipe issues one instruction fewer per pair.
__device__ __forceinline__ void relu_fma2_mixed(float2& acc, uint32_t x0, uint32_t x1, float w0, float w1) {
  asm("{\n\t"
      ".reg .f32 a, b;\n\t"
      ".reg .b64 p, q, r;\n\t"
      "fma.rn.sat.f32 a, %2, 0f33000000, 0f00000000;\n\t"
      "max.f32 b, %3, 0f00000000;\n\t"
      "mov.b64 p, {a, b};\n\t"
      "mov.b64 q, {%4, %5};\n\t"
      "mov.b64 r, {%0, %1};\n\t"
      "fma.rn.f32x2 r, p, q, r;\n\t"
      "mov.b64 {%0, %1}, r;\n\t"
      "}"
      : "+f"(acc.x), "+f"(acc.y)
      : "f"(__uint_as_float(x0)), "f"(__uint_as_float(x1)), "f"(w0), "f"(w1));
}

// Shared-memory struct at the first 1024-byte boundary of the dynamic shared
// buffer, reached by pointer arithmetic on the buffer itself so that the
// compiler keeps the shared address space (ld.shared, not generic loads).
template <typename T>
__device__ __forceinline__ T& smem_aligned_1024(unsigned char* raw) {
  return *reinterpret_cast<T*>(raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u));
}

// Predicated global stores (one instruction, no branch around them).
__device__ __forceinline__ void st_f32_if(float* p, float v, bool pred) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.f32 [%0], %1;\n\t}" ::"l"(p), "f"(v),
               "r"(static_cast<int>(pred))
               : "memory");
}
__device__ __forceinline__ void st_u32_if(uint32_t* p, uint32_t v, bool pred) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.u32 [%0], %1;\n\t}" ::"l"(p), "r"(v),
               "r"(static_cast<int>(pred))
               : "memory");
}

// Named barrier over `count` threads (a subset of the CTA).
__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, fp8 e4m3 x e4m3 -> f32, both K-major.
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives (once) on `bar` when every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Issues a 32-column TMEM load; the registers are valid only after tmem_ld_wait()
// followed by tmem_reg_fence(r) (which makes every later use depend on the wait).
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32-column TMEM load and its wait in one statement: the registers are
// defined only after the wait, so no separate register fence is needed.
__device__ __forceinline__ void tmem_ld_x32_sync(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_reg_fence(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

// Shared-memory matrix descriptor of a K-major operand tile stored as rows of
// 128 bytes with the 128-byte swizzle (the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B); 8-row groups are 1024 bytes apart.  The tile
// base must be 1024-byte aligned.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(1) << 16;                      // leading byte offset (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;              // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1) << 46;                      // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                      // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f8f6f4, A = B = E4M3, D = F32, K-major A and B.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int M, int N) {
  return (1u << 4)                                  // D format F32
         | (0u << 7) | (0u << 10)                   // A, B = E4M3
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

}  // namespace hcu

// Per-translation-unit sticky status word (no relocatable device code), its
// reader and the setter of the unit's wait limit.
#define HCU_DEFINE_STATUS(accessor)                                                        \
  static __device__ unsigned int g_hcu_status;                                             \
  namespace hcu {                                                                          \
  cudaError_t accessor##_set_wait_limit(uint64_t ns) {                                     \
    return cudaMemcpyToSymbol(g_hcu_wait_limit_ns, &ns, sizeof(ns));                       \
  }                                                                                        \
  cudaError_t accessor(uint32_t* out, int clear) {                                         \
    unsigned int v = 0;                                                                    \
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_hcu_status, sizeof(v));                     \
    if (e != cudaSuccess) return e;                                                        \
    *out |= v;                                                                             \
    if (clear && v) {                                                                      \
      const unsigned int z = 0;                                                            \
      e = cudaMemcpyToSymbol(g_hcu_status, &z, sizeof(z));                                 \
    }                                                                                      \
    return e;                                                                              \
  }                                                                                        \
  }

namespace hcu {
// Internal host helpers shared by the translation units (capi.cu).
void set_last_error(cudaError_t e);
void set_last_error_msg(const char* a, const char* b);
int launch_status();  // HCU_OK or HCU_ERR_LAUNCH from cudaGetLastError()
int sm_count();       // SM count of the current device (cached per device)
cudaError_t status_dequant(uint32_t* out, int clear);
cudaError_t status_topk(uint32_t* out, int clear);
cudaError_t status_logits(uint32_t* out, int clear);
cudaError_t status_mla(uint32_t* out, int clear);
cudaError_t status_dequant_set_wait_limit(uint64_t ns);
cudaError_t status_topk_set_wait_limit(uint64_t ns);
cudaError_t status_logits_set_wait_limit(uint64_t ns);
cudaError_t status_mla_set_wait_limit(uint64_t ns);
}  // namespace hcu
