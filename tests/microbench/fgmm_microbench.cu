// Microbenchmarks behind the tensor-core E-step's design (sm_100a).
//
// Measures, with many operations in flight and one wait at the end:
//   * tcgen05.mma throughput (cycles per instruction) for kind::f16 and
//     kind::tf32, M = 64 / 128 (cta_group::1) and M = 256 (cta_group::2),
//     N = 64 .. 256, A from shared memory or from TMEM, optionally while the
//     other warps of the CTA stream shared memory (contention);
//   * MUFU ex2 (f32 and f16x2) and FFMA issue rates per SM;
//   * co-resident clusters of 2 .. 16 CTAs at a given shared-memory size
//     (host occupancy query).
// Every wait is bounded (~2 s); a timeout sets *err and the kernel returns.
// Built as its own shared library (build_microbench.py); not part of the
// product library.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr long long kTimeout = 4000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int* err) {
  const long long t0 = clock64();
  while (!mbar_try(b, parity)) {
    if (clock64() - t0 > kTimeout) {
      atomicOr(err, 1);
      return false;
    }
  }
  return true;
}
// UMMA shared-memory descriptor, K-major, 128-byte swizzle (SBO = 1024 B).
__device__ __forceinline__ uint64_t desc_k(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}
// Instruction descriptor: fp32 accumulate, A/B format fmt (0 f16, 2 tf32),
// both K-major.
__device__ __forceinline__ uint32_t idesc(int M, int N, int fmt) {
  return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

template <bool TF32, bool ATMEM>
__device__ __forceinline__ void mma1(uint32_t d, uint64_t adesc, uint32_t atmem, uint64_t bdesc,
                                     uint32_t id, uint32_t acc) {
  if constexpr (ATMEM) {
    if constexpr (TF32)
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
          "r"(atmem), "l"(bdesc), "r"(id), "r"(acc)
          : "memory");
    else
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
          "r"(atmem), "l"(bdesc), "r"(id), "r"(acc)
          : "memory");
  } else {
    if constexpr (TF32)
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
          "l"(adesc), "l"(bdesc), "r"(id), "r"(acc)
          : "memory");
    else
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
          "l"(adesc), "l"(bdesc), "r"(id), "r"(acc)
          : "memory");
  }
}

constexpr int kABytes = 128 * 128;   // 128 rows x 128 B (one 128B-swizzle K chunk)
constexpr int kBBytes = 256 * 128;   // 256 rows x 128 B
constexpr int kHammerBytes = 64 * 1024;
constexpr int kSmemBytes = 1024 + kABytes + kBBytes + kHammerBytes;

struct __align__(8) Ctl {
  uint64_t bar;
  uint32_t tmem;
  volatile int done;
};

// One CTA per SM, 128 threads.  Thread 0 issues `iters` (a multiple of 4) MMAs (M, N, K = 16
// f16 or K = 8 tf32) into one accumulator, then commits and waits.  With
// `hammer`, warps 1-3 stream 16-byte shared loads and stores over a separate
// 64 KB region until the MMAs are done and report the bytes moved.
// out[3 * cta] = {cycles from first issue to completion, issue cycles,
// hammer bytes}.
template <bool TF32, bool ATMEM>
__global__ void __launch_bounds__(128, 1)
    mma_rate_kernel(int iters, int M, int N, int hammer, long long* out, int* err) {
  extern __shared__ uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                           ~uintptr_t(1023));
  uint8_t* As = sm;
  uint8_t* Bs = sm + kABytes;
  uint8_t* Hs = Bs + kBBytes;
  __shared__ Ctl ctl;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // operands: small finite values (fp16 or tf32 bit patterns)
  for (int i = threadIdx.x; i < (kABytes + kBBytes) / 4; i += blockDim.x) {
    uint32_t v;
    if (TF32) {
      v = __float_as_uint(0.125f * (float)((i * 37) % 7 - 3));
    } else {
      const __half h0 = __float2half(0.125f * (float)((i * 37) % 7 - 3));
      const __half h1 = __float2half(0.0625f * (float)((i * 11) % 5 - 2));
      v = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
    }
    reinterpret_cast<uint32_t*>(sm)[i] = v;
  }
  if (threadIdx.x == 0) {
    mbar_init(&ctl.bar, 1);
    ctl.done = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(&ctl.tmem))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = ctl.tmem;
  const uint32_t acol = 256;  // A in TMEM: columns 256.. (32 columns = 4 K-steps of f16)
  if (ATMEM) {
    // each warp writes its 32 lanes of the A region
    uint32_t v = TF32 ? __float_as_uint(0.25f) : 0x34003400u;
    for (int c = 0; c < 32; ++c) {
      const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + acol + c;
      asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(ta), "r"(v)
                   : "memory");
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

  if (threadIdx.x == 0) {
    const uint32_t id = idesc(M, N, TF32 ? 2 : 0);
    uint64_t ad[4], bd[4];
    for (int s = 0; s < 4; ++s) {
      ad[s] = desc_k(smem_u32(As) + 32 * s);
      bd[s] = desc_k(smem_u32(Bs) + 32 * s);
    }
    const long long t0 = clock64();
    for (int i = 0; i < iters; i += 4) {
#pragma unroll
      for (int s = 0; s < 4; ++s)
        mma1<TF32, ATMEM>(tmem, ad[s], tmem + acol + 8 * s, bd[s], id, (i + s) > 0 ? 1u : 0u);
    }
    const long long t1 = clock64();
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(&ctl.bar))
        : "memory");
    mbar_wait(&ctl.bar, 0, err);
    const long long t2 = clock64();
    ctl.done = 1;
    out[3 * blockIdx.x + 0] = t2 - t0;
    out[3 * blockIdx.x + 1] = t1 - t0;
  } else if (hammer && warp >= 1) {
    // 96 threads stream 16-byte loads and stores until the MMAs finish
    long long bytes = 0;
    uint4 acc = make_uint4(0, 0, 0, 0);
    const int t = threadIdx.x - 32;
    const long long t0 = clock64();
    for (int it = 0; it < (1 << 22) && !ctl.done; ++it) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int off = ((it * 8 + u) * 96 + t) % (kHammerBytes / 16);
        uint4* p = reinterpret_cast<uint4*>(Hs) + off;
        const uint4 v = *p;
        acc.x ^= v.x; acc.y += v.y;
        *reinterpret_cast<uint4*>(Hs + ((off + 7) % (kHammerBytes / 16)) * 16) = acc;
      }
      bytes += 8 * 32;
      if (clock64() - t0 > kTimeout) break;
    }
    if (lane == 0) atomicAdd(reinterpret_cast<unsigned long long*>(&out[3 * blockIdx.x + 2]),
                             (unsigned long long)(bytes * 32));
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

// cta_group::2: a cluster of 2 CTAs; the even CTA issues M = 256 MMAs with
// A rows 0-127 from its own shared memory and 128-255 from the peer's, and B
// columns split between the two (N/2 each); the commit arrives on both CTAs'
// barrier.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1)
    mma_rate_2cta_kernel(int iters, int N, long long* out, int* err) {
  extern __shared__ uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                           ~uintptr_t(1023));
  uint8_t* As = sm;
  uint8_t* Bs = sm + kABytes;
  __shared__ Ctl ctl;
  const int warp = threadIdx.x >> 5;
  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  for (int i = threadIdx.x; i < (kABytes + kBBytes) / 4; i += blockDim.x) {
    const __half h0 = __float2half(0.125f * (float)((i * 37) % 7 - 3));
    reinterpret_cast<uint32_t*>(sm)[i] =
        (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h0) << 16);
  }
  if (threadIdx.x == 0) {
    mbar_init(&ctl.bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(&ctl.tmem))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = ctl.tmem;
  if (rank == 0 && threadIdx.x == 0) {
    const uint32_t id = idesc(256, N, 0);
    uint64_t ad[4], bd[4];
    for (int s = 0; s < 4; ++s) {
      ad[s] = desc_k(smem_u32(As) + 32 * s);
      bd[s] = desc_k(smem_u32(Bs) + 32 * s);
    }
    const long long t0 = clock64();
    for (int i = 0; i < iters; i += 4)
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
          "l"(ad[s]), "l"(bd[s]), "r"(id), "r"((i + s) > 0 ? 1u : 0u)
          : "memory");
    }
    const long long t1 = clock64();
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(&ctl.bar))
        : "memory");
    mbar_wait(&ctl.bar, 0, err);
    const long long t2 = clock64();
    out[3 * (blockIdx.x / 2) + 0] = t2 - t0;
    out[3 * (blockIdx.x / 2) + 1] = t1 - t0;
  }
  // the odd CTA stays in the cluster barrier below until the even CTA has
  // seen its MMAs (which read this CTA's shared memory) complete
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

// Issue-rate kernel: every thread runs `iters` rounds of 8 independent
// operations of kind `op` (0 ex2.approx.ftz.f32, 1 ex2.approx.f16x2,
// 2 fma.rn.f32, 3 two ex2.f32 and six FFMA, 4 redux.sync.add.u32,
// 5 redux.sync.max.f32, 6 shfl.sync.bfly, 7 ex2.approx.ftz.f32 predicated
// on for lane 0 of each warp only, 8 the same predicated off on every lane).
// out[cta] = cycles.
__global__ void __launch_bounds__(1024, 1) issue_rate_kernel(int iters, int op, long long* out,
                                                             float* sink) {
  float v[8];
  uint32_t h[8];
  for (int i = 0; i < 8; ++i) {
    v[i] = -0.001f * (float)(threadIdx.x + i);
    h[i] = 0xBC00BC00u ^ (uint32_t)(threadIdx.x + i);
  }
  __syncthreads();
  const long long t0 = clock64();
  if (op == 0) {
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 8; ++i) asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(v[i]));
  } else if (op == 1) {
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 8; ++i) asm volatile("ex2.approx.f16x2 %0, %0;" : "+r"(h[i]));
  } else if (op == 2) {
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        asm volatile("fma.rn.f32 %0, %0, 0f3F7FF000, 0f3A800000;" : "+f"(v[i]));
  } else if (op == 4) {
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        asm volatile("redux.sync.add.u32 %0, %0, 0xffffffff;" : "+r"(h[i]));
  } else if (op == 5) {
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        asm volatile("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(v[i]));
  } else if (op == 7 || op == 8) {
    const uint32_t on = op == 7 ? ((threadIdx.x & 31) == 0 ? 1u : 0u) : 0u;
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %1, 0;\n\t@p ex2.approx.ftz.f32 %0, %0;\n\t}"
                     : "+f"(v[i])
                     : "r"(on));
  } else if (op == 6) {
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        asm volatile("shfl.sync.bfly.b32 %0, %0, 16, 0x1f, 0xffffffff;" : "+r"(h[i]));
  } else {
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int i = 0; i < 2; ++i) asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(v[i]));
#pragma unroll
      for (int i = 2; i < 8; ++i)
        asm volatile("fma.rn.f32 %0, %0, 0f3F7FF000, 0f3A800000;" : "+f"(v[i]));
    }
  }
  __syncthreads();
  const long long t1 = clock64();
  float s = 0.f;
  for (int i = 0; i < 8; ++i) s += v[i] + __half2float(__ushort_as_half((unsigned short)h[i]));
  if (s == 12345.f) sink[threadIdx.x] = s;
  if (threadIdx.x == 0) out[blockIdx.x] = t1 - t0;
}

__global__ void cluster_probe_kernel() {}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int fgmm_mb_smem_bytes(void) { return kSmemBytes; }

// kind: 0 f16 A smem, 1 f16 A tmem, 2 tf32 A smem, 3 tf32 A tmem.
__attribute__((visibility("default"))) int fgmm_mb_mma_rate(int kind, int ctas, int iters,
                                                            int M, int N, int hammer,
                                                            long long* out_dev, int* err_dev,
                                                            void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  switch (kind) {
    case 0:
      e = cudaFuncSetAttribute(mma_rate_kernel<false, false>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e == cudaSuccess)
        mma_rate_kernel<false, false><<<ctas, 128, kSmemBytes, s>>>(iters, M, N, hammer, out_dev,
                                                                    err_dev);
      break;
    case 1:
      e = cudaFuncSetAttribute(mma_rate_kernel<false, true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e == cudaSuccess)
        mma_rate_kernel<false, true><<<ctas, 128, kSmemBytes, s>>>(iters, M, N, hammer, out_dev,
                                                                   err_dev);
      break;
    case 2:
      e = cudaFuncSetAttribute(mma_rate_kernel<true, false>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e == cudaSuccess)
        mma_rate_kernel<true, false><<<ctas, 128, kSmemBytes, s>>>(iters, M, N, hammer, out_dev,
                                                                   err_dev);
      break;
    case 3:
      e = cudaFuncSetAttribute(mma_rate_kernel<true, true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e == cudaSuccess)
        mma_rate_kernel<true, true><<<ctas, 128, kSmemBytes, s>>>(iters, M, N, hammer, out_dev,
                                                                  err_dev);
      break;
    default:
      return -1;
  }
  if (e != cudaSuccess) return (int)e;
  return (int)cudaGetLastError();
}

// cta_group::2, M = 256; `pairs` clusters of 2 CTAs.
__attribute__((visibility("default"))) int fgmm_mb_mma_rate_2cta(int pairs, int iters, int N,
                                                                 long long* out_dev,
                                                                 int* err_dev, void* stream) {
  cudaError_t e = cudaFuncSetAttribute(mma_rate_2cta_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return (int)e;
  mma_rate_2cta_kernel<<<2 * pairs, 128, kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(
      iters, N, out_dev, err_dev);
  return (int)cudaGetLastError();
}

__attribute__((visibility("default"))) int fgmm_mb_issue_rate(int ctas, int threads, int iters,
                                                              int op, long long* out_dev,
                                                              float* sink_dev, void* stream) {
  issue_rate_kernel<<<ctas, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      iters, op, out_dev, sink_dev);
  return (int)cudaGetLastError();
}

// Largest number of co-resident clusters of `cluster` CTAs (threads each,
// smem_bytes dynamic shared memory) of a trivial kernel.
__attribute__((visibility("default"))) int fgmm_mb_max_clusters(int cluster, int threads,
                                                                int smem_bytes) {
  cudaFuncSetAttribute(cluster_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       smem_bytes);
  if (cluster > 8)
    cudaFuncSetAttribute(cluster_probe_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(cluster * 64, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  cudaError_t e = cudaOccupancyMaxActiveClusters(&n, cluster_probe_kernel, &cfg);
  return e == cudaSuccess ? n : -(int)e;
}

}  // extern "C"
