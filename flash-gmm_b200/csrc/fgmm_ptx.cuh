// PTX helpers shared by the tcgen05 kernels of libflashgmm_sm100 (sm_100a):
// mbarriers with bounded waits, bulk copies, tcgen05 MMA / TMEM access,
// UMMA shared-memory descriptors, fp16 hi/lo splitting and exact
// power-of-two scaling.
#pragma once

#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

namespace fgmm {
namespace {

constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 2 GHz

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_cluster(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; returns false (and raises the abort flag) on timeout or when
// another role of this CTA already aborted.  `code` is OR-ed into *err on
// timeout so the host can tell which wait gave up.
template <bool kCluster = false>
__device__ __forceinline__ bool mbar_wait_flag(uint64_t* b, uint32_t parity,
                                               volatile int* abort_flag, int* err, int code) {
  const uint32_t a = smem_u32(b);
  if (kCluster ? mbar_try_cluster(a, parity) : mbar_try(a, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (kCluster ? mbar_try_cluster(a, parity) : mbar_try(a, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kTimeoutCycles) {
      *abort_flag = 1;
      atomicOr(err, code);
      return false;
    }
  }
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_cta(uint32_t local_addr, uint32_t cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(cta));
  return r;
}
// Asynchronous remote store that completes `bytes` on the destination mbarrier.
__device__ __forceinline__ void st_async_f2(uint32_t addr, float a, float b, uint32_t bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
          addr),
      "f"(a), "f"(b), "r"(bar)
      : "memory");
}
// Bulk copy global -> this CTA's shared memory, completing `bytes` on `bar`.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(b))
               : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]; kind::f16 with fp16 inputs, fp32 accum.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The same MMA with the B descriptor given as its two 32-bit words: callers
// keep the constant high word and add byte offsets >> 4 to the low word (the
// start-address field, bits 0-13, does not carry for shared-memory offsets),
// so each MMA of an unrolled sequence costs one integer add to set up.
__device__ __forceinline__ void mma_ts2(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo,
                                        uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 bd;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 bd, {%2, %3};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %4, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}
// mma_ss with both descriptors given by their low words and one shared high
// word (both K-major, or both with the same swizzle, SBO and version bits).
__device__ __forceinline__ void mma_ss2(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo,
                                        uint32_t d_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 ad, bd;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 ad, {%1, %3};\n\t"
      "mov.b64 bd, {%2, %3};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %4, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(d_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}
// True on exactly one active lane of the warp (all 32 lanes must call it).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}
// D[tmem] (+)= A[smem desc] * B[smem desc]; kind::f16 with fp16 inputs, fp32 accum.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 16 lanes x 256 bits, 4 repetitions along the columns: thread t holds,
// for repetition j (columns 8j..8j+7), lanes base + t/4 and base + 8 + t/4 at
// columns 8j + 2(t%4) and 8j + 2(t%4) + 1:
//   v[4j] = (t/4, c), v[4j+1] = (t/4, c+1), v[4j+2] = (8+t/4, c), v[4j+3] = (8+t/4, c+1).
__device__ __forceinline__ void tmem_ld16x256_x4(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}
// One column (one 32-bit value per lane) at a run-time column address.
__device__ __forceinline__ uint32_t tmem_ld1(uint32_t taddr) {
  uint32_t v;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v) : "r"(taddr) : "memory");
  return v;
}
__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float redux_max(float v) {
  float r;
  asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float lg2(float x) {
  float r;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// Pack (lo_elem, hi_elem) as f16x2 with lo_elem in the low half.
__device__ __forceinline__ uint32_t pack_f16(float lo_elem, float hi_elem) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi_elem), "f"(lo_elem));
  return r;
}
__device__ __forceinline__ float f16lo_f(uint32_t p) {
  return __half2float(__ushort_as_half((unsigned short)(p & 0xffffu)));
}
__device__ __forceinline__ float f16hi_f(uint32_t p) {
  return __half2float(__ushort_as_half((unsigned short)(p >> 16)));
}

// Split (a, b) into an fp16 hi pair and an fp16 lo pair:
// a = hi.x + lo.x + O(2^-22 |a|) for |a| in fp16's normal range.
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_f16(a, b);
  lo = pack_f16(a - f16lo_f(hi), b - f16hi_f(hi));
}

// UMMA shared-memory descriptors (sm_100: version bits 46-47 = 1), 128B swizzle.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}
// Words of desc_kmajor / desc_mnmajor: low word for a shared-memory address,
// and the constant high word (SBO = 1024 B, version 1, 128B swizzle).
__device__ __forceinline__ uint32_t desc_lo_kmajor(uint32_t addr) {
  return ((addr >> 4) & 0x3FFFu) | (1u << 16);
}
__device__ __forceinline__ uint32_t desc_lo_mnmajor(uint32_t addr, uint32_t chunk_bytes) {
  return ((addr >> 4) & 0x3FFFu) | ((chunk_bytes >> 4) << 16);
}
constexpr uint32_t kDescHi = 64u | (1u << 14) | (2u << 29);
// MN-major: LBO = byte stride between 64-element chunks along N.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t addr, uint32_t chunk_bytes) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(chunk_bytes >> 4) << 16) |
         (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: f16 x f16 -> f32 (c_format = 1,
// a_format = b_format = 0), M = 128.
__host__ __device__ constexpr uint32_t idesc_f16(int N, bool b_mn_major) {
  return (1u << 4) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}

// Byte offset of element (row, feature) inside one stage's hi (or lo) buffer:
// chunk = feature/64 (rows*128 bytes each), 128 B per row, 16B-granule XOR
// swizzle.
__device__ __forceinline__ uint32_t xoff(int row, int f, int chunk_bytes) {
  const int e = f & 63;
  return (uint32_t)((f >> 6) * chunk_bytes + row * 128 + ((((e >> 3) ^ (row & 7))) << 4) +
                    ((e & 7) << 1));
}

// ---------------------------------------------------------------------------
// Power-of-two scale exponent e such that m 2^-e lies in [2^(t-1), 2^t);
// 0 for m == 0.  Exact scaling keeps fp16 hi/lo splits in their normal range.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int scale_exp_to(float m, int t) {
  if (!(m > 0.f) || !isfinite(m)) return 0;
  int e;
  frexpf(m, &e);  // m = f * 2^e, f in [0.5, 1)
  return e - t;
}
__device__ __forceinline__ int scale_exp(float m) { return scale_exp_to(m, 5); }
// X scale of each family: iso maps max|mu| into [16, 32); diag maps
// max|mu - c| into [4, 8), leaving room for the squared features.
template <bool DIAG>
__device__ __forceinline__ int x_scale_exp(float m) {
  return scale_exp_to(m, DIAG ? 3 : 5);
}


}  // namespace
}  // namespace fgmm
