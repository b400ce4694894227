// Tensor-core (tcgen05 / TMEM) full-covariance E-step for sm_100a, D <= 64.
//
// The reference evaluates the Mahalanobis term with one (BLOCK_N x D) x
// (D x D) dot per component and d2 slice (flash_gmm_full_h100.py:71-139) and
// accumulates sig_outer with per-d2 outer products and atomics (full:146-228).
// Here the E-step is two tensor-core passes plus small set-up / reduction
// kernels:
//
// Pass 1 (full_ll_kernel, rows on TMEM lanes): for a 128-row tile of
//   x~ = x - c (c = mean of the means), V = x~ L_k is evaluated per region of
//   16 components x 16 columns j of their L's: one M=128, N=256 GEMM with
//   A = the x~ tile and B = those L columns, both fp16 hi/lo in shared memory
//   (three passes lo*hi + hi*lo + hi*hi, 22-bit operands).  L_k is lower
//   triangular, so columns j in block jb only meet rows d >= 16 jb: region jb
//   runs the K-steps s = jb .. Dp/16-1 (at D = 64: 10 of 16 K-steps).
//   The epilogue (thread = row) forms v = V - b_k (b_k = (mu_k - c)^T L_k),
//   maha = |v|^2, ll2 = const_k - maha/2 * log2 e (full:124-129, 289-296, log2
//   units), keeps an online log-sum-exp per row and writes ll2 for pass 2.
//   Two accumulators (2 x 256 TMEM columns) let the MMAs of group g+1 run
//   while the epilogue drains group g.
//
// Pass 2 (full_stats_kernel, components on TMEM lanes): per 64-row chunk,
//   T[k, f] += sum_n r_nk z_nf with z = [x~_i x~_j (i <= j), x~_i, 1] laid out
//   in quads of 4 columns (2244 columns at D = 64; mu_acc and Nk come from the
//   same GEMM).  A = R^T
//   (fp16 hi/lo written to TMEM from ll2 and logZ), B = the z chunk (fp16
//   hi/lo, generated on chip from x~ into the MN-major shared-memory layout),
//   N = 256 features per CTA.  CTAs tile (feature block, component block,
//   row slab); partials are reduced in slab order (deterministic).
//
// Every wait is bounded (timeout -> error word -> NaN outputs).
#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>
#include <type_traits>

#include "fgmm_internal.cuh"
#include "fgmm_ptx.cuh"

namespace fgmm {
namespace {

constexpr int kFullMaxD = 64;
constexpr int kSmsFull = 148;

// ---- pass 1
constexpr int kP1Rows = 128;
constexpr int kP1EpiWarps = 16;              // four warps per TMEM lane quadrant
constexpr int kP1LoadWarp = 16;
constexpr int kP1MmaWarp = 17;
constexpr int kP1Threads = 18 * 32;
constexpr int kP1LStages = 2;
constexpr int kXTile = kP1Rows * 128;        // 16 KB: one hi (or lo) x~ tile, 64 features
constexpr int kCG = 16;                      // components per group (16 x 16 columns = MMA N)
constexpr int kLGroup = 256 * 128;           // 32 KB: one hi (or lo) region of L columns
constexpr int kP1BSlots = 2;                 // ring of per-group b vectors + constants
constexpr int kBOff = kCG * kFullMaxD * 4;   // 4 KB: b of 16 components, then 16 float2
constexpr int kBSlot = kBOff + kCG * 8;

// ---- pass 2
constexpr int kP2Rows = 64;                  // rows per chunk (MMA K extent)
constexpr int kP2Feat = 256;                 // features per CTA (MMA N)
constexpr int kP2Comps = 128;                // components per CTA (MMA M)
constexpr int kP2ZWarps = 16;                // warps 0-15: z chunks (4 rows each)
constexpr int kP2LoadWarp = 16;
constexpr int kP2MmaWarp = 17;
constexpr int kP2Threads = 18 * 32;
constexpr int kZChunk = kP2Rows * 128;       // 8 KB: 64 rows x 64 features (fp16)
constexpr int kZStage = 2 * 4 * kZChunk;     // hi + lo, 256 features: 64 KB
constexpr int kRBlock = kP2Comps * 128;      // 16 KB: R^T hi (or lo), 128 components x 64 rows

struct P1Params {
  const uint8_t* xsplit;   // [num_tiles][hi 16 KB | lo 16 KB]  x~ 2^-a1, swizzled K-major
  const uint8_t* lgroups;  // [num_groups][Dp/16 regions][hi 32 KB | lo 32 KB] L columns
                           // 2^-s_k, K-major; region row i*16 + jj = column 16 jb + jj of
                           // component 16 g + i
  const float* bvec;       // [Kpad][Dp]  b_k = (mu_k - c)^T L_k
  const float2* kconst;    // [num_groups][16]  {const_k in log2 units, s_k}
  const int* amax;         // max|mu - c| (float bits) -> a1
  int64_t N;
  int K, Dp, num_groups, num_tiles;
  int64_t ld_ll;           // row stride of ll2 (= num_tiles * 128)
  float* ll2;              // [Kpad][ld_ll]
  float* lz2;              // [ld_ll]  logZ in log2 units (for pass 2)
  float* logZ;             // [N]      natural log
  int* err;
};

struct __align__(8) P1Ctl {
  uint64_t xfull[2], xempty[2];
  uint64_t bfull[kP1BSlots], bempty[kP1BSlots];
  uint64_t lfull[kP1LStages], lempty[kP1LStages];
  uint64_t afull[2], aempty[2];
  uint64_t lse_bar;
  uint32_t tmem_base;
  volatile int abort_flag;
};

struct P2Params {
  const uint8_t* rt;       // [chunks][ncb][hi 16 KB | lo 16 KB]  R^T, K-major swizzled
  const float* xs2;        // [Npad][D+1]  x~ 2^-a2 and a constant 1
  int64_t N;
  int D, nf, nfb, ncb, slabs;
  int64_t rows_per_slab;   // multiple of 64
  float* part;             // [slabs][ncb*128][nfb*256]
  int* err;
};

struct __align__(8) P2Ctl {
  // x rows (consumed by the z warps) and R^T (consumed by the MMAs) have
  // their own barriers, so the next x rows load as soon as a z chunk is built
  uint64_t xin_full[2], xin_empty[2], rin_full[2], rin_empty[2], zfull[2], zempty[2], tdone;
  uint32_t tmem_base;
  volatile int abort_flag;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ---------------------------------------------------------------------------
// Prep, one block per component k < Kpad (64 threads; thread e = output index):
//   s_k from max|L_k| (exact power of two), region layout of the L columns
//   (row (k % 16)*16 + e % 16 of region e/16 of group k/16 holds L_k[:, e]
//   2^-s_k, fp16 hi/lo),
//   b_k[e] = sum_d (mu_kd - c_d) L_k[d, e],
//   const_k = (log pi_k + sum_d log(|L_kdd| + 1e-30) - D/2 log 2pi) log2 e.
// Components >= K get zero columns and const = -1e30.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(64) full_prep_kernel(
    const float* __restrict__ mu, int64_t smk, int64_t smd, const float* __restrict__ L,
    const float* __restrict__ lpi, const float* __restrict__ cvec, int K, int D, int Dp,
    uint8_t* __restrict__ lgroups, float* __restrict__ bvec, float2* __restrict__ kconst) {
  const int k = blockIdx.x;
  const int e = threadIdx.x;
  const bool valid = k < K;
  const bool col = valid && e < D;
  const float* Lk = L + (size_t)k * D * D;
  float lmax = 0.f;
  double b = 0.0, logd = 0.0;
  if (col) {
    for (int d = 0; d < D; ++d) {
      const float v = Lk[(size_t)d * D + e];
      lmax = fmaxf(lmax, fabsf(v));
      b += ((double)mu[(int64_t)k * smk + (int64_t)d * smd] - (double)cvec[d]) * (double)v;
    }
    logd = log(fabs((double)Lk[(size_t)e * D + e]) + 1e-30);
  }
  __shared__ float s_max[2];
  __shared__ double s_logd[2];
  for (int o = 16; o > 0; o >>= 1) {
    lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    logd += __shfl_xor_sync(0xffffffffu, logd, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s_max[threadIdx.x >> 5] = lmax;
    s_logd[threadIdx.x >> 5] = logd;
  }
  __syncthreads();
  const int sk = scale_exp_to(fmaxf(s_max[0], s_max[1]), 5);
  if (e < Dp) {
    uint8_t* grp = lgroups + ((size_t)(k / kCG) * (Dp / 16) + e / 16) * 2 * kLGroup;
    const int rr = (k % kCG) * 16 + e % 16;
    for (int d0 = 0; d0 < 64; d0 += 8) {
      uint32_t hi[4], lo[4];
      for (int u = 0; u < 8; u += 2) {
        const float v0 = (col && d0 + u < D) ? ldexpf(Lk[(size_t)(d0 + u) * D + e], -sk) : 0.f;
        const float v1 =
            (col && d0 + u + 1 < D) ? ldexpf(Lk[(size_t)(d0 + u + 1) * D + e], -sk) : 0.f;
        split2(v0, v1, hi[u / 2], lo[u / 2]);
      }
      const uint32_t off = xoff(rr, d0, kLGroup);
      *reinterpret_cast<uint4*>(grp + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(grp + kLGroup + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    bvec[(size_t)k * Dp + e] = col ? (float)b : 0.f;
  }
  if (threadIdx.x == 0) {
    double c = -1e30;
    if (valid) {
      c = ((double)lpi[k] + s_logd[0] + s_logd[1] - 0.5 * D * kLog2Pi) * kLog2E;
      if (!(c > -1e30)) c = -1e30;
    }
    kconst[k] = make_float2((float)c, (float)sk);
  }
}

// Row stride (floats) of the pass-2 x~ rows: D values, the constant 1, zeros,
// even (8-byte aligned pairs) and covering every j-quad.
__host__ __device__ __forceinline__ int xs2_stride(int D) {
  const int need = D + 2 > 4 * ((D + 3) / 4) ? D + 2 : 4 * ((D + 3) / 4);
  return (need + 1) & ~1;
}

// Split pass (any X strides): a half-warp per row, lane l of the half
// carries features 4l..4l+3 (features >= D and rows >= N are zero); each warp
// takes 8 consecutive rows per step and issues all their loads first:
//   xsplit: x~ 2^-a1 as fp16 hi/lo in 128-row swizzled K-major tiles (pass 1);
//   xs2:    x~ 2^-a2 in fp32, D values then a constant 1 per row (pass 2).
constexpr int kFullSplitRows = 8;
template <class TX>
__global__ void __launch_bounds__(256) full_split_kernel(
    const TX* __restrict__ X, int64_t sxn, int64_t sxd, int vec_ok, int64_t N, int D,
    int64_t rows_pad, const float* __restrict__ cvec, const int* __restrict__ amax,
    uint8_t* __restrict__ xsplit, float* __restrict__ xs2, int* __restrict__ err) {
  const int lane = threadIdx.x & 31, hw = lane >> 4, l16 = lane & 15;
  const float am = __int_as_float(*amax);
  const int a1 = scale_exp_to(am, 5), a2 = scale_exp_to(am, 3);
  const int f = 4 * l16;  // 64 features per half-warp
  const int xs_stride = xs2_stride(D);
  float4 cc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (f + 0 < D) cc.x = cvec[f + 0];
  if (f + 1 < D) cc.y = cvec[f + 1];
  if (f + 2 < D) cc.z = cvec[f + 2];
  if (f + 3 < D) cc.w = cvec[f + 3];
  // rows_pad is a multiple of 128, so every row of a step is < rows_pad
  for (int64_t row0 = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * kFullSplitRows;
       row0 < rows_pad; row0 += (int64_t)gridDim.x * 8 * kFullSplitRows) {
    float4 xr[kFullSplitRows / 2];
#pragma unroll
    for (int u = 0; u < kFullSplitRows / 2; ++u) {
      const int64_t row = row0 + 2 * u + hw;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row < N) {
        const TX* src = X + row * sxn;
        if (vec_ok && f + 3 < D) {
          x = ldx4(src + f);
        } else {
          if (f + 0 < D) x.x = ldx(src + (int64_t)(f + 0) * sxd);
          if (f + 1 < D) x.y = ldx(src + (int64_t)(f + 1) * sxd);
          if (f + 2 < D) x.z = ldx(src + (int64_t)(f + 2) * sxd);
          if (f + 3 < D) x.w = ldx(src + (int64_t)(f + 3) * sxd);
        }
      }
      xr[u] = x;
    }
#pragma unroll
    for (int u = 0; u < kFullSplitRows / 2; ++u) {
      const int64_t row = row0 + 2 * u + hw;
      float4 x = xr[u];
      if (row < N) {
        x.x = f + 0 < D ? x.x - cc.x : 0.f;
        x.y = f + 1 < D ? x.y - cc.y : 0.f;
        x.z = f + 2 < D ? x.z - cc.z : 0.f;
        x.w = f + 3 < D ? x.w - cc.w : 0.f;
      }
      float* x2row = xs2 + row * xs_stride;
      if (l16 == 0) {  // constant slot D, zeros up to the stride
        x2row[D] = 1.0f;
        for (int d = D + 1; d < xs_stride; ++d) x2row[d] = 0.f;
      }
      const float4 x2 = make_float4(ldexpf(x.x, -a2), ldexpf(x.y, -a2), ldexpf(x.z, -a2),
                                    ldexpf(x.w, -a2));
      if (f + 0 < D) x2row[f + 0] = x2.x;
      if (f + 1 < D) x2row[f + 1] = x2.y;
      if (f + 2 < D) x2row[f + 2] = x2.z;
      if (f + 3 < D) x2row[f + 3] = x2.w;
      // products of two such values must stay inside fp16's range in pass 2
      if (!(fmaxf(fmaxf(fabsf(x2.x), fabsf(x2.y)), fmaxf(fabsf(x2.z), fabsf(x2.w))) < 255.f))
        atomicOr(err, 0x20000);
      x = make_float4(ldexpf(x.x, -a1), ldexpf(x.y, -a1), ldexpf(x.z, -a1), ldexpf(x.w, -a1));
      const float mx = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
      if (!(mx < 65504.f)) atomicOr(err, 0x10000);  // outside fp16 range (or NaN)
      uint32_t h0, l0, h1, l1;
      split2(x.x, x.y, h0, l0);
      split2(x.z, x.w, h1, l1);
      uint8_t* tile = xsplit + (row / kP1Rows) * (2 * kXTile);
      const uint32_t off = xoff((int)(row % kP1Rows), f, kXTile);
      *reinterpret_cast<uint2*>(tile + off) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(tile + kXTile + off) = make_uint2(l0, l1);
    }
  }
}

// ---------------------------------------------------------------------------
// Pass 1: distances, per-row log-sum-exp, ll2 for pass 2.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kP1Threads, 1) full_ll_kernel(const P1Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* xs = smem;                                         // [2][hi | lo] x~ tiles
  uint8_t* lsm = smem + 4 * kXTile;                           // [stages][hi | lo] L groups
  float2* red = reinterpret_cast<float2*>(lsm + kP1LStages * 2 * kLGroup);  // [2][2][4][128]
  uint8_t* bst = reinterpret_cast<uint8_t*>(red + 16 * kP1Rows);            // [slots][kBSlot]
  P1Ctl* ctl = reinterpret_cast<P1Ctl*>(bst + kP1BSlots * kBSlot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = (p.num_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  volatile int* abort_flag = &ctl->abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->xfull[i], 1);
      mbar_init(&ctl->xempty[i], 1);
      mbar_init(&ctl->afull[i], 1);
      mbar_init(&ctl->aempty[i], kP1EpiWarps);
    }
    for (int i = 0; i < kP1LStages; ++i) {
      mbar_init(&ctl->lfull[i], 1);
      mbar_init(&ctl->lempty[i], 1);
    }
    mbar_init(&ctl->lse_bar, kP1EpiWarps);
    for (int i = 0; i < kP1BSlots; ++i) {
      mbar_init(&ctl->bfull[i], 1);
      mbar_init(&ctl->bempty[i], kP1EpiWarps);
    }
    ctl->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(&ctl->tmem_base))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int xa = scale_exp_to(__int_as_float(*p.amax), 5);

  // Tiles of this CTA: blockIdx.x + i * gridDim.x, processed in pairs (2q, 2q+1):
  // each L group is loaded once per pair and multiplied with both x~ tiles,
  // the two products alternating between the two TMEM accumulators.
  const int npairs = (ntiles + 1) / 2;
  auto pair_tiles = [&](int q) -> int { return 2 * q + 1 < ntiles ? 2 : 1; };
  auto tile_of = [&](int q, int tt) -> int64_t {
    return (int64_t)blockIdx.x + (int64_t)(2 * q + tt) * gridDim.x;
  };

  const int nreg = p.Dp / 16;  // regions (column blocks) per component group
  if (warp == kP1MmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(256, false);
      int gi = 0, li = 0;  // accumulator uses, region loads
      bool ok = true;
      for (int q = 0; q < npairs && ok; ++q) {
        const int nt = pair_tiles(q);
        for (int tt = 0; tt < nt && ok; ++tt)
          ok = mbar_wait_flag(&ctl->xfull[tt], q & 1, abort_flag, p.err, 1);
        for (int g = 0; g < p.num_groups && ok; ++g) {
          for (int jb = 0; jb < nreg && ok; ++jb, ++li) {
            const int st = li % kP1LStages;
            if (!mbar_wait_flag(&ctl->lfull[st], (li / kP1LStages) & 1, abort_flag, p.err, 2)) {
              ok = false;
              break;
            }
            const uint32_t lhi = smem_u32(lsm + st * 2 * kLGroup), llo = lhi + kLGroup;
            for (int tt = 0; tt < nt; ++tt, ++gi) {
              const int acc = gi & 1;
              if (!mbar_wait_flag(&ctl->aempty[acc], ((gi >> 1) & 1) ^ 1, abort_flag, p.err, 4)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t xhi = smem_u32(xs + tt * 2 * kXTile);
              const uint32_t dxh = desc_lo_kmajor(xhi), dxl = desc_lo_kmajor(xhi + kXTile);
              const uint32_t dlh = desc_lo_kmajor(lhi), dll = desc_lo_kmajor(llo);
              const uint32_t dacc = tmem + (uint32_t)(acc * 256);
              // terms x_lo*L_hi, x_hi*L_lo, x_hi*L_hi (smallest magnitudes first);
              // K-steps below jb meet the zero upper triangle of L and are skipped.
              // Descriptor words advance 32 bytes (2 in >> 4 units) per K-step;
              // each K-step count is issued straight-line.
              auto p1_mma = [&](int term, int ks, uint32_t accf) {
                mma_ss2(dacc, (term == 0 ? dxl : dxh) + 2u * (uint32_t)ks,
                        (term == 1 ? dll : dlh) + 2u * (uint32_t)ks, kDescHi, idesc, accf);
              };
              auto tri = [&](auto nkc) {
                constexpr int NK = decltype(nkc)::value;
#pragma unroll
                for (int term = 0; term < 3; ++term)
#pragma unroll
                  for (int i = 0; i < NK; ++i)
                    p1_mma(term, jb + i, (term == 0 && i == 0) ? 0u : 1u);
              };
              switch (nreg - jb) {
                case 4: tri(std::integral_constant<int, 4>{}); break;
                case 3: tri(std::integral_constant<int, 3>{}); break;
                case 2: tri(std::integral_constant<int, 2>{}); break;
                case 1: tri(std::integral_constant<int, 1>{}); break;
                default:
                  for (int term = 0; term < 3; ++term)
                    for (int ks = jb; ks < nreg; ++ks)
                      p1_mma(term, ks, (term == 0 && ks == jb) ? 0u : 1u);
              }
              tc_commit(&ctl->afull[acc]);
            }
            tc_commit(&ctl->lempty[st]);
          }
        }
        for (int tt = 0; tt < nt; ++tt) tc_commit(&ctl->xempty[tt]);
      }
    }
    __syncwarp();
  } else if (warp == kP1LoadWarp) {
    if (lane == 0) {
      int li = 0, bi = 0;
      bool ok = true;
      const uint32_t bbytes = (uint32_t)(kCG * p.Dp * 4);
      for (int q = 0; q < npairs && ok; ++q) {
        const int nt = pair_tiles(q);
        for (int tt = 0; tt < nt && ok; ++tt) {
          if (!mbar_wait_flag(&ctl->xempty[tt], (q & 1) ^ 1, abort_flag, p.err, 8)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&ctl->xfull[tt], 2 * kXTile);
          bulk_g2s(smem_u32(xs + tt * 2 * kXTile), p.xsplit + tile_of(q, tt) * (2 * kXTile),
                   2 * kXTile, &ctl->xfull[tt]);
        }
        for (int g = 0; g < p.num_groups && ok; ++g, ++bi) {
          const int bs = bi % kP1BSlots;
          if (!mbar_wait_flag(&ctl->bempty[bs], ((bi / kP1BSlots) & 1) ^ 1, abort_flag, p.err,
                              128)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&ctl->bfull[bs], bbytes + (uint32_t)(kCG * 8));
          bulk_g2s(smem_u32(bst + bs * kBSlot), p.bvec + (size_t)g * kCG * p.Dp, bbytes,
                   &ctl->bfull[bs]);
          bulk_g2s(smem_u32(bst + bs * kBSlot + kBOff), p.kconst + (size_t)g * kCG,
                   (uint32_t)(kCG * 8), &ctl->bfull[bs]);
          for (int jb = 0; jb < nreg; ++jb, ++li) {
            const int st = li % kP1LStages;
            if (!mbar_wait_flag(&ctl->lempty[st], ((li / kP1LStages) & 1) ^ 1, abort_flag, p.err,
                                16)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&ctl->lfull[st], 2 * kLGroup);
            bulk_g2s(smem_u32(lsm + st * 2 * kLGroup),
                     p.lgroups + ((size_t)g * nreg + jb) * (2 * kLGroup), 2 * kLGroup,
                     &ctl->lfull[st]);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp < kP1EpiWarps) {
    // thread = row (TMEM lane) of tile tt; warp quarter h takes components
    // i = h, h+4, h+8, h+12 of each group (16 columns of each per region) and
    // keeps their partial |v|^2 over the regions
    const int q4 = warp & 3, h = warp >> 2;
    const int row = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const float kHalfLog2E = 0.72134752044448170f;
    int gi = 0, bi = 0;
    for (int q = 0; q < npairs; ++q) {
      const int nt = pair_tiles(q);
      float m[2] = {-3.0e38f, -3.0e38f}, l[2] = {0.f, 0.f};
      bool ok = true;
      for (int g = 0; g < p.num_groups && ok; ++g, ++bi) {
        const int bs = bi % kP1BSlots;
        if (!mbar_wait_flag(&ctl->bfull[bs], (bi / kP1BSlots) & 1, abort_flag, p.err, 256)) {
          ok = false;
          break;
        }
        const float* bgrp = reinterpret_cast<const float*>(bst + bs * kBSlot);
        const float2* kgrp = reinterpret_cast<const float2*>(bst + bs * kBSlot + kBOff);
        float sc[4];  // V = V' 2^(a1 + s_k)
#pragma unroll
        for (int u = 0; u < 4; ++u) sc[u] = ldexpf(1.0f, xa + (int)kgrp[h + 4 * u].y);
        float mp[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // partial |v|^2
        for (int jb = 0; jb < nreg && ok; ++jb) {
#pragma unroll
          for (int tt = 0; tt < 2; ++tt) {
            if (tt >= nt) break;
            const int acc = gi & 1;
            if (!mbar_wait_flag(&ctl->afull[acc], (gi >> 1) & 1, abort_flag, p.err, 32)) {
              ok = false;
              break;
            }
            ++gi;
            tc_fence_after();
#pragma unroll
            for (int u0 = 0; u0 < 4; u0 += 2) {
              uint32_t v[32];
              tmem_ld16(tmem + lane_base + acc * 256 + (h + 4 * u0) * 16, v);
              tmem_ld16(tmem + lane_base + acc * 256 + (h + 4 * u0 + 4) * 16, v + 16);
              float bb[32];
#pragma unroll
              for (int w = 0; w < 2; ++w) {
                const float4* bk =
                    reinterpret_cast<const float4*>(bgrp + (h + 4 * (u0 + w)) * p.Dp + 16 * jb);
#pragma unroll
                for (int z = 0; z < 4; ++z) {
                  const float4 b4 = bk[z];
                  bb[16 * w + 4 * z + 0] = b4.x;
                  bb[16 * w + 4 * z + 1] = b4.y;
                  bb[16 * w + 4 * z + 2] = b4.z;
                  bb[16 * w + 4 * z + 3] = b4.w;
                }
              }
              tmem_wait_ld();
#pragma unroll
              for (int w = 0; w < 2; ++w) {
                float s0 = 0.f, s1 = 0.f;
#pragma unroll
                for (int z = 0; z < 16; z += 2) {
                  const float d0 = fmaf(__uint_as_float(v[16 * w + z]), sc[u0 + w], -bb[16 * w + z]);
                  const float d1 =
                      fmaf(__uint_as_float(v[16 * w + z + 1]), sc[u0 + w], -bb[16 * w + z + 1]);
                  s0 = fmaf(d0, d0, s0);
                  s1 = fmaf(d1, d1, s1);
                }
                mp[tt][u0 + w] += s0 + s1;
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->aempty[acc]);
          }
        }
        if (!ok) break;
#pragma unroll
        for (int tt = 0; tt < 2; ++tt) {
          if (tt >= nt) break;
          const int64_t n = tile_of(q, tt) * kP1Rows + row;
          const bool live = n < p.N;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int k = g * kCG + h + 4 * u;
            if (k >= p.K) break;
            const float ll2 = fmaf(-kHalfLog2E, mp[tt][u], kgrp[h + 4 * u].x);
            if (ll2 > m[tt]) {
              l[tt] = fmaf(l[tt], ex2(m[tt] - ll2), 1.0f);
              m[tt] = ll2;
            } else {
              l[tt] += ex2(ll2 - m[tt]);
            }
            if (live) p.ll2[(size_t)k * p.ld_ll + n] = ll2;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->bempty[bs]);
      }
      if (!ok) break;
      // combine the four quarters of each row; red double-buffered by pair parity
      float2* rq = red + (q & 1) * 8 * kP1Rows;
      for (int tt = 0; tt < nt; ++tt) rq[(tt * 4 + h) * kP1Rows + row] = make_float2(m[tt], l[tt]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->lse_bar);
      if (!mbar_wait_flag(&ctl->lse_bar, q & 1, abort_flag, p.err, 64)) break;
      if (h == 0) {
        for (int tt = 0; tt < nt; ++tt) {
          float2 o[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) o[u] = rq[(tt * 4 + u) * kP1Rows + row];
          const float M = fmaxf(fmaxf(o[0].x, o[1].x), fmaxf(o[2].x, o[3].x));
          const float Ls = (o[0].y * ex2(o[0].x - M) + o[1].y * ex2(o[1].x - M)) +
                           (o[2].y * ex2(o[2].x - M) + o[3].y * ex2(o[3].x - M));
          const float lz2 = M + lg2(Ls);
          const int64_t n = tile_of(q, tt) * kP1Rows + row;
          if (n < p.N) {
            p.logZ[n] = lz2 * 0.6931471805599453f;
            p.lz2[n] = lz2;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

// Pass-2 features come in quads of 4 consecutive columns:
//   pair quad (i, q):  x~_i x~_j for j = 4q..4q+3, q >= floor(i/4)  (covers i <= j;
//                      the few j < i columns are extra and ignored)
//   x quad q:          x~_j for j = 4q..4q+3            (mu_acc)
//   one quad:          [1, 0, 0, 0]                      (Nk)
//   zero quads pad the last feature block.
// With Dq = ceil(D/4), pair quads of row i start at pairbase(i) =
// i*Dq - sum_{i'<i} floor(i'/4).  Columns for j >= D are never read back.
__host__ __device__ __forceinline__ int quad_dq(int D) { return (D + 3) / 4; }
__host__ __device__ __forceinline__ int pairbase(int i, int Dq) {
  const int a = i >> 2, b = i & 3;
  return i * Dq - (2 * a * (a - 1) + a * b);
}
__host__ __device__ __forceinline__ int pair_quads(int D) { return pairbase(D, quad_dq(D)); }
__host__ __device__ __forceinline__ int num_features(int D) {
  return 4 * (pair_quads(D) + quad_dq(D) + 1);
}
// Feature column of x_i x_j (i <= j), of x_i, and of the constant.
__host__ __device__ __forceinline__ int pair_feature(int i, int j, int D) {
  const int Dq = quad_dq(D);
  return 4 * (pairbase(i, Dq) + (j >> 2) - (i >> 2)) + (j & 3);
}
__host__ __device__ __forceinline__ int x_feature(int i, int D) {
  return 4 * (pair_quads(D) + (i >> 2)) + (i & 3);
}
__host__ __device__ __forceinline__ int one_feature(int D) {
  return 4 * (pair_quads(D) + quad_dq(D));
}
// Kind of quad Q: 0 pair (i, q), 1 x quad (q), 2 one, 3 zero; packed as
// kind | i << 8 | q << 16.
__device__ __forceinline__ uint32_t quad_desc(int Q, int D) {
  const int Dq = quad_dq(D), P = pair_quads(D);
  if (Q < P) {
    int i = 0;
    while (i + 1 < D && pairbase(i + 1, Dq) <= Q) ++i;
    const int q = (i >> 2) + (Q - pairbase(i, Dq));
    return 0u | ((uint32_t)i << 8) | ((uint32_t)q << 16);
  }
  if (Q < P + Dq) return 1u | ((uint32_t)(Q - P) << 16);
  if (Q == P + Dq) return 2u;
  return 3u;
}

// ---------------------------------------------------------------------------
// Responsibilities for pass 2, one block per (64-row chunk, component block),
// thread = component: r = 2^(ll2 - lz2) (0 past N or K), split into fp16
// hi/lo and written as the K-major, 128B-swizzled A operand of pass 2 (one
// 128-byte row of 64 rows per component).  The 32 KB block is built in
// shared memory and written out with coalesced 16-byte stores.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kP2Comps) full_resp_kernel(const float* __restrict__ ll2,
                                                             int64_t ld_ll,
                                                             const float* __restrict__ lz2,
                                                             int64_t N, int K, int ncb,
                                                             uint8_t* __restrict__ rt) {
  const int chunk = (int)blockIdx.x / ncb, cbk = (int)blockIdx.x % ncb;
  const int t = threadIdx.x;
  const int k = cbk * kP2Comps + t;
  const int64_t r0 = (int64_t)chunk * kP2Rows;
  __shared__ float lz[kP2Rows];
  __shared__ __align__(16) uint8_t img[2 * kRBlock];
  if (t < kP2Rows) lz[t] = r0 + t < N ? lz2[r0 + t] : 0.f;
  __syncthreads();
  const bool kvalid = k < K;
  const float* llk = ll2 + (size_t)(kvalid ? k : 0) * ld_ll + r0;
  uint8_t* blk = rt + ((size_t)chunk * ncb + cbk) * (2 * kRBlock);
  float rv[kP2Rows];
  if (kvalid && r0 + kP2Rows <= N) {
    float4 v4[kP2Rows / 4];
#pragma unroll
    for (int u = 0; u < kP2Rows / 4; ++u) v4[u] = __ldg(reinterpret_cast<const float4*>(llk) + u);
#pragma unroll
    for (int u = 0; u < kP2Rows / 4; ++u) {
      rv[4 * u + 0] = ex2(v4[u].x - lz[4 * u + 0]);
      rv[4 * u + 1] = ex2(v4[u].y - lz[4 * u + 1]);
      rv[4 * u + 2] = ex2(v4[u].z - lz[4 * u + 2]);
      rv[4 * u + 3] = ex2(v4[u].w - lz[4 * u + 3]);
    }
  } else {
#pragma unroll
    for (int u = 0; u < kP2Rows; ++u)
      rv[u] = (kvalid && r0 + u < N) ? ex2(llk[u] - lz[u]) : 0.f;
  }
#pragma unroll
  for (int g = 0; g < kP2Rows / 8; ++g) {
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) split2(rv[8 * g + 2 * u], rv[8 * g + 2 * u + 1], hi[u], lo[u]);
    const uint32_t off = xoff(t, 8 * g, kRBlock);
    *reinterpret_cast<uint4*>(img + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(img + kRBlock + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
  __syncthreads();
#pragma unroll 4
  for (int i = t; i < 2 * kRBlock / 16; i += kP2Comps)
    reinterpret_cast<uint4*>(blk)[i] = reinterpret_cast<const uint4*>(img)[i];
}

// ---------------------------------------------------------------------------
// Pass 2: T[k, f] = sum_n r_nk z_nf for one (feature block, component block,
// row slab) per CTA.  Per 64-row chunk one loader lane bulk-copies the x~
// rows (64 x (D+1) floats) and another R^T (32 KB), each double-buffered on
// its own barriers; 16 warps build the z chunk; one thread issues the MMAs
// (A = R^T, B = z, both from shared memory).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kP2Threads, 1) full_stats_kernel(const P2Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int xs_stride = xs2_stride(p.D);
  const uint32_t xs_bytes = (uint32_t)(kP2Rows * xs_stride * 4);
  uint8_t* rst = smem;                                        // [2][hi | lo] R^T, 32 KB each
  uint8_t* zst = smem + 4 * kRBlock;                          // [2][hi | lo] z, 64 KB each
  float* xst = reinterpret_cast<float*>(zst + 2 * kZStage);   // [2][64][D+1]
  P2Ctl* ctl = reinterpret_cast<P2Ctl*>(xst + 2 * kP2Rows * xs_stride);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int fb = (int)blockIdx.x % p.nfb;
  const int cbk = ((int)blockIdx.x / p.nfb) % p.ncb;
  const int slab = (int)blockIdx.x / (p.nfb * p.ncb);
  const int64_t row_begin = (int64_t)slab * p.rows_per_slab;
  const int64_t row_end = p.N < row_begin + p.rows_per_slab ? p.N : row_begin + p.rows_per_slab;
  const int nchunks =
      row_end > row_begin ? (int)((row_end - row_begin + kP2Rows - 1) / kP2Rows) : 0;
  volatile int* abort_flag = &ctl->abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->xin_full[i], 1);
      mbar_init(&ctl->xin_empty[i], kP2ZWarps);  // z warps
      mbar_init(&ctl->rin_full[i], 1);
      mbar_init(&ctl->rin_empty[i], 1);          // MMA commit
      mbar_init(&ctl->zfull[i], kP2ZWarps);
      mbar_init(&ctl->zempty[i], 1);
    }
    mbar_init(&ctl->tdone, 1);
    ctl->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(
                     smem_u32(&ctl->tmem_base))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == kP2LoadWarp) {
    // lane 0 streams the x rows, lane 1 the R^T blocks
    if (lane < 2) {
      for (int c = 0; c < nchunks; ++c) {
        const int b = c & 1;
        const int64_t r0 = row_begin + (int64_t)c * kP2Rows;
        const int64_t chunk = r0 / kP2Rows;
        if (lane == 0) {
          if (!mbar_wait_flag(&ctl->xin_empty[b], ((c >> 1) & 1) ^ 1, abort_flag, p.err, 1)) break;
          mbar_arrive_expect_tx(&ctl->xin_full[b], xs_bytes);
          bulk_g2s(smem_u32(xst + b * kP2Rows * xs_stride), p.xs2 + r0 * xs_stride, xs_bytes,
                   &ctl->xin_full[b]);
        } else {
          if (!mbar_wait_flag(&ctl->rin_empty[b], ((c >> 1) & 1) ^ 1, abort_flag, p.err, 1)) break;
          mbar_arrive_expect_tx(&ctl->rin_full[b], 2 * kRBlock);
          bulk_g2s(smem_u32(rst + b * 2 * kRBlock),
                   p.rt + ((size_t)chunk * p.ncb + cbk) * (2 * kRBlock), 2 * kRBlock,
                   &ctl->rin_full[b]);
        }
      }
    }
    __syncwarp();
  } else if (warp == kP2MmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kP2Feat, true);  // A K-major, B MN-major
      for (int c = 0; c < nchunks; ++c) {
        const int b = c & 1;
        if (!mbar_wait_flag(&ctl->zfull[b], (c >> 1) & 1, abort_flag, p.err, 2) ||
            !mbar_wait_flag(&ctl->rin_full[b], (c >> 1) & 1, abort_flag, p.err, 4))
          break;
        tc_fence_after();
        const uint32_t rhi = smem_u32(rst + b * 2 * kRBlock);
        const uint32_t zhi = smem_u32(zst + b * kZStage);
        const uint32_t drh = desc_lo_kmajor(rhi), drl = desc_lo_kmajor(rhi + kRBlock);
        const uint32_t dzh = desc_lo_mnmajor(zhi, kZChunk);
        const uint32_t dzl = desc_lo_mnmajor(zhi + 4 * kZChunk, kZChunk);
        // terms r_lo*z_hi, r_hi*z_lo, r_hi*z_hi, straight-line; K-step s: R^T
        // 32 bytes along the row, z 16 rows = 2048 bytes
#pragma unroll
        for (int term = 0; term < 3; ++term) {
#pragma unroll
          for (int s = 0; s < kP2Rows / 16; ++s)
            mma_ss2(tmem, (term == 0 ? drl : drh) + 2u * (uint32_t)s,
                    (term == 1 ? dzl : dzh) + (uint32_t)(s * (2048 >> 4)), kDescHi, idesc,
                    (c == 0 && term == 0 && s == 0) ? 0u : 1u);
        }
        tc_commit(&ctl->zempty[b]);
        tc_commit(&ctl->rin_empty[b]);
      }
      tc_commit(&ctl->tdone);
    }
    __syncwarp();
  } else {
    // ---- z chunks: warp zw builds rows 4zw..4zw+3; lane l owns the feature
    // quads lane and 32 + lane of this CTA's 64 (features 4l.. and 128+4l..)
    const int zw = warp;
    uint32_t qd[2];
    qd[0] = quad_desc(fb * (kP2Feat / 4) + lane, p.D);
    qd[1] = quad_desc(fb * (kP2Feat / 4) + 32 + lane, p.D);
    int c = 0;
    for (; c < nchunks; ++c) {
      const int b = c & 1;
      if (!mbar_wait_flag(&ctl->xin_full[b], (c >> 1) & 1, abort_flag, p.err, 8) ||
          !mbar_wait_flag(&ctl->zempty[b], ((c >> 1) & 1) ^ 1, abort_flag, p.err, 16))
        break;
      const float* xsb = xst + b * kP2Rows * xs_stride;
      uint8_t* zs = zst + b * kZStage;
#pragma unroll 1
      for (int rr = 0; rr < 4; ++rr) {
        const int r = zw * 4 + rr;
        const float* xr = xsb + r * xs_stride;
#pragma unroll
        for (int grp = 0; grp < 2; ++grp) {
          const uint32_t d = qd[grp];
          const uint32_t kind = d & 0xffu;
          float z[4];
          if (kind <= 1u) {
            const int j0 = 4 * (int)(d >> 16);
            const float2 a01 = *reinterpret_cast<const float2*>(xr + j0);
            const float2 a23 = *reinterpret_cast<const float2*>(xr + j0 + 2);
            const float xi = kind == 0u ? xr[(d >> 8) & 0xffu] : 1.0f;
            z[0] = xi * a01.x;
            z[1] = xi * a01.y;
            z[2] = xi * a23.x;
            z[3] = xi * a23.y;
          } else {
            z[0] = kind == 2u ? 1.0f : 0.f;
            z[1] = 0.f;
            z[2] = 0.f;
            z[3] = 0.f;
          }
          uint32_t h0, l0, h1, l1;
          split2(z[0], z[1], h0, l0);
          split2(z[2], z[3], h1, l1);
          const uint32_t off = xoff(r, grp * 128 + 4 * lane, kZChunk);
          *reinterpret_cast<uint2*>(zs + off) = make_uint2(h0, h1);
          *reinterpret_cast<uint2*>(zs + 4 * kZChunk + off) = make_uint2(l0, l1);
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&ctl->zfull[b]);
        mbar_arrive(&ctl->xin_empty[b]);
      }
    }
    // partial statistics of this CTA -> workspace: warp (quadrant q, quarter h)
    // reads TMEM lanes 32q.. and columns 64h..64h+63
    const int q = warp & 3, h = warp >> 2;
    const int kl = q * 32 + lane;
    const int ldp = p.nfb * kP2Feat;
    float* out = p.part + ((size_t)slab * p.ncb * kP2Comps + (size_t)cbk * kP2Comps + kl) * ldp +
                 (size_t)fb * kP2Feat + 64 * h;
    const bool ok = c == nchunks && mbar_wait_flag(&ctl->tdone, 0, abort_flag, p.err, 32);
    if (nchunks > 0 && ok) {
      tc_fence_after();
      for (int blk = 0; blk < 2; ++blk) {
        uint32_t tv[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + 64 * h + 32 * blk, tv);
        tmem_wait_ld();
        float4* o4 = reinterpret_cast<float4*>(out + 32 * blk);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          o4[u] = make_float4(__uint_as_float(tv[4 * u]), __uint_as_float(tv[4 * u + 1]),
                              __uint_as_float(tv[4 * u + 2]), __uint_as_float(tv[4 * u + 3]));
      }
    } else {
      const float v = nchunks > 0 ? __int_as_float(0x7fc00000) : 0.f;
      for (int f = 0; f < 64; ++f) out[f] = v;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
  }
}

// Sum the pass-2 partials over slabs (in order) and undo the centring and
// scaling:  Nk = S1,  mu_acc = Sx 2^a2 + c Nk,
//   sig_outer[i][j] = Sxx[min(i,j)][max(i,j)] 2^(2 a2) + c_i mu~_j + mu~_i c_j
//                     + Nk c_i c_j        (mu~ = Sx 2^a2, uncentred: full:213-228)
// NaN everywhere on a device-side error.
__global__ void __launch_bounds__(256) full_reduce_kernel(
    const float* __restrict__ part, int slabs, int Kp, int ldp, int K, int D,
    const float* __restrict__ cvec, const int* __restrict__ amax, const int* __restrict__ err,
    float* __restrict__ Nk, float* __restrict__ mu_acc, float* __restrict__ sig, int accumulate) {
  // one block per component: its Nk and mu~ (sums over slabs) once in shared
  // memory, then every sig_outer element from its pair feature
  const int k = blockIdx.x;
  const int a2 = scale_exp_to(__int_as_float(*amax), 3);
  const double s1 = ldexp(1.0, a2), s2 = ldexp(1.0, 2 * a2);
  const bool bad = *err != 0;
  const float qnan = __int_as_float(0x7fc00000);
  auto feat_sum = [&](int f) -> double {
    double s = 0.0;
    for (int sl = 0; sl < slabs; ++sl) s += part[((size_t)sl * Kp + k) * ldp + f];
    return s;
  };
  __shared__ double s_m[kFullMaxD], s_n;
  for (int i = threadIdx.x; i <= D; i += blockDim.x) {
    if (i < D) s_m[i] = feat_sum(x_feature(i, D)) * s1;
    else s_n = feat_sum(one_feature(D));
  }
  __syncthreads();
  const double n = s_n;
  const int per_k = D * D + D + 1;
  for (int w = threadIdx.x; w < per_k; w += blockDim.x) {
    if (w == D * D + D) {
      const float v = bad ? qnan : (float)n;
      Nk[k] = accumulate ? Nk[k] + v : v;
    } else if (w >= D * D) {
      const int i = w - D * D;
      const float v = bad ? qnan : (float)(s_m[i] + (double)cvec[i] * n);
      float* dst = mu_acc + (size_t)k * D + i;
      *dst = accumulate ? *dst + v : v;
    } else {
      const int i = w / D, j = w % D;
      const int a = min(i, j), b = max(i, j);
      const double sxx = feat_sum(pair_feature(a, b, D)) * s2;
      const double ci = cvec[i], cj = cvec[j];
      const float v = bad ? qnan : (float)(sxx + ci * s_m[j] + s_m[i] * cj + n * ci * cj);
      float* dst = sig + (size_t)k * D * D + w;
      *dst = accumulate ? *dst + v : v;
    }
  }
}

struct FullPlan {
  int Dp, num_groups, Kpad, num_tiles, nf, nfb, ncb, slabs;
  int64_t Npad, rows_per_slab;
};

FullPlan plan_full(int64_t N, int K, int D) {
  FullPlan pl;
  pl.Dp = (D + 15) / 16 * 16;
  pl.num_groups = (K + kCG - 1) / kCG;
  pl.Kpad = pl.num_groups * kCG;
  pl.num_tiles = (int)((N + kP1Rows - 1) / kP1Rows);
  pl.Npad = (int64_t)pl.num_tiles * kP1Rows;
  pl.nf = num_features(D);
  pl.nfb = (pl.nf + kP2Feat - 1) / kP2Feat;
  pl.ncb = (K + kP2Comps - 1) / kP2Comps;
  const int64_t nch_total = (N + kP2Rows - 1) / kP2Rows;
  pl.slabs = (int)std::max<int64_t>(1, std::min<int64_t>(kSmsFull / (pl.nfb * pl.ncb), nch_total));
  pl.rows_per_slab = ((nch_total + pl.slabs - 1) / pl.slabs) * kP2Rows;
  return pl;
}

size_t p1_smem_bytes() {
  return 1024 + (size_t)4 * kXTile + (size_t)kP1LStages * 2 * kLGroup +
         (size_t)16 * kP1Rows * sizeof(float2) + (size_t)kP1BSlots * kBSlot + sizeof(P1Ctl) + 64;
}
size_t p2_smem_bytes(int D) {
  return 1024 + (size_t)4 * kRBlock + (size_t)2 * kZStage +
         (size_t)2 * kP2Rows * xs2_stride(D) * 4 + sizeof(P2Ctl) + 16;
}

struct FullWs {
  int* err;
  float* cvec;
  uint8_t* lgroups;
  float* bvec;
  float2* kconst;
  uint8_t* xsplit;
  float* xs2;
  float* ll2;
  float* lz2;
  uint8_t* rt;
  float* part;
  size_t bytes;
};

FullWs carve_full(void* base, const FullPlan& pl, int D) {
  WsCarve w(base);
  FullWs ws;
  ws.err = w.take<int>(64);
  ws.cvec = w.take<float>(kFullMaxD);
  ws.lgroups = w.take<uint8_t>((size_t)pl.num_groups * (pl.Dp / 16) * 2 * kLGroup);
  ws.bvec = w.take<float>((size_t)pl.Kpad * pl.Dp);
  ws.kconst = w.take<float2>((size_t)pl.num_groups * 16);
  ws.xsplit = w.take<uint8_t>((size_t)pl.num_tiles * 2 * kXTile);
  ws.xs2 = w.take<float>((size_t)pl.Npad * xs2_stride(D));
  ws.ll2 = w.take<float>((size_t)pl.Kpad * pl.Npad);
  ws.lz2 = w.take<float>((size_t)pl.Npad);
  ws.rt = w.take<uint8_t>((size_t)(pl.Npad / kP2Rows) * pl.ncb * 2 * kRBlock);
  ws.part = w.take<float>((size_t)pl.slabs * pl.ncb * kP2Comps * pl.nfb * kP2Feat);
  ws.bytes = w.used + 256;
  return ws;
}

}  // namespace

bool full_tc_supported(const EstepArgs& a) {
  if (a.D > kFullMaxD || a.N <= 0) return false;
  const FullPlan pl = plan_full(a.N, a.K, a.D);
  return (double)pl.Kpad * (double)pl.Npad * 4.0 <= 8.0e9;  // ll2 scratch bound
}

size_t full_tc_workspace_bytes(int64_t N, int K, int D) {
  EstepArgs probe{};
  probe.N = N;
  probe.K = K;
  probe.D = D;
  if (K < 1 || !full_tc_supported(probe)) return 0;
  return carve_full(nullptr, plan_full(N, K, D), D).bytes;
}

cudaError_t full_tc_estep(const EstepArgs& a) {
  const FullPlan pl = plan_full(a.N, a.K, a.D);
  const FullWs ws = carve_full(a.ws, pl, a.D);
  cudaStream_t st = a.stream;
  // err[0]: device error word; err[1]: max|mu - c| (float bits)
  cudaError_t e = cudaMemsetAsync(ws.err, 0, 2 * sizeof(int), st);
  if (e != cudaSuccess) return e;
  int* amax = ws.err + 1;
  launch_centre(a, pl.Dp, ws.cvec, amax, st);
  full_prep_kernel<<<pl.Kpad, 64, 0, st>>>(a.mu, a.smk, a.smd, a.cov, a.lpi, ws.cvec, a.K, a.D,
                                           pl.Dp, ws.lgroups, ws.bvec, ws.kconst);
  const int vec_ok = a.x_vec_ok();
  const int sblocks =
      (int)std::min<int64_t>((pl.Npad + 8 * kFullSplitRows - 1) / (8 * kFullSplitRows),
                             16 * kSmsFull);
  with_xtype(a.xtype, [&](auto tx) {
    using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
    full_split_kernel<TX><<<sblocks, 256, 0, st>>>(a.x<TX>(), a.sxn, a.sxd, vec_ok, a.N, a.D,
                                                   pl.Npad, ws.cvec, amax, ws.xsplit, ws.xs2,
                                                   ws.err);
    return 0;
  });

  P1Params p1;
  p1.xsplit = ws.xsplit;
  p1.lgroups = ws.lgroups;
  p1.bvec = ws.bvec;
  p1.kconst = ws.kconst;
  p1.amax = amax;
  p1.N = a.N;
  p1.K = a.K;
  p1.Dp = pl.Dp;
  p1.num_groups = pl.num_groups;
  p1.num_tiles = pl.num_tiles;
  p1.ld_ll = pl.Npad;
  p1.ll2 = ws.ll2;
  p1.lz2 = ws.lz2;
  p1.logZ = a.logZ;
  p1.err = ws.err;
  const size_t sm1 = p1_smem_bytes();
  e = ensure_dynamic_smem(reinterpret_cast<const void*>(full_ll_kernel), sm1);
  if (e != cudaSuccess) return e;
  profile_mark(false, st);
  full_ll_kernel<<<std::min(pl.num_tiles, kSmsFull), kP1Threads, sm1, st>>>(p1);

  const int nchunk_total = (int)((a.N + kP2Rows - 1) / kP2Rows);
  full_resp_kernel<<<nchunk_total * pl.ncb, kP2Comps, 0, st>>>(ws.ll2, pl.Npad, ws.lz2, a.N, a.K,
                                                                pl.ncb, ws.rt);
  P2Params p2;
  p2.rt = ws.rt;
  p2.xs2 = ws.xs2;
  p2.N = a.N;
  p2.D = a.D;
  p2.nf = pl.nf;
  p2.nfb = pl.nfb;
  p2.ncb = pl.ncb;
  p2.slabs = pl.slabs;
  p2.rows_per_slab = pl.rows_per_slab;
  p2.part = ws.part;
  p2.err = ws.err;
  const size_t sm2 = p2_smem_bytes(a.D);
  e = ensure_dynamic_smem(reinterpret_cast<const void*>(full_stats_kernel), sm2);
  if (e != cudaSuccess) return e;
  full_stats_kernel<<<pl.nfb * pl.ncb * pl.slabs, kP2Threads, sm2, st>>>(p2);
  profile_mark(true, st);

  full_reduce_kernel<<<a.K, 256, 0, st>>>(ws.part, pl.slabs, pl.ncb * kP2Comps,
                                              pl.nfb * kP2Feat, a.K, a.D, ws.cvec, amax, ws.err,
                                              a.Nk, a.mu_acc, a.sig, (a.flags & 1u) ? 1 : 0);
  count_launches(7);
  return cudaGetLastError();
}

}  // namespace fgmm
