// Tensor-core (tcgen05 / TMEM) E-step for sm_100a: isotropic and diagonal
// covariance.
//
// One fused kernel replaces the reference's two launches per family (online
// LSE pass + statistics pass: flash_gmm.py:50-103 / 110-166, and
// flash_gmm_diag_h100.py:63-130 / 159-282): the distance GEMM is evaluated
// ONCE per (row, component) pair and the responsibilities never leave the
// chip.
//
// Both families are the same computation over a per-row feature vector F:
//   isotropic:  F = x - c                 (nfeat = Dp; c = mean of the mu's)
//               ll2[k,n] = c0'_k - ish_k |x_n-c|^2 + sum_d 2 ish_k (mu_kd-c_d) F_nd
//   diagonal:   F = [(x-c)^2, (x-c)]      (nfeat = 2 Dp)
//               ll2[k,n] = c0'_k + sum_d (-A_kd (x-c)_d^2 + B_kd (x-c)_d)
//               A = 1/2 e^{-lss} log2 e,  B = 2 A (mu - c)
// (log2 units: the folding of flash_gmm_h100.py:286-291 / 137-138 and
// flash_gmm_diag_h100.py:332-339 / 116-119).  The statistics GEMM
// T = R^T F gives sum r (x-c) (iso; mu_acc = T + c Nk) or
// [sum r (x-c)^2, sum r (x-c)] (diag), from which the reduction forms
// sig = rxsq - 2 m mu + m^2 Nk (diag:258-260).  Centring by one global vector
// leaves every distance unchanged and shrinks the magnitudes that cancel in
// the expanded form when the data sit away from the origin.
//
// Orientation ("components on TMEM lanes"):
//   * a CTA owns a slice of 128 components = the 128 TMEM lanes; a cluster of
//     C = ceil(K/128) CTAs covers all components and processes the same
//     row tiles of F in lock-step (128 rows iso, 64 rows diag: TMEM holds
//     T nfeat | S rows | R^T rows | W nfeat columns = 512 at most);
//   * distance GEMM  S^T[k, n] = sum_f W[k, f] F[n, f]
//       A = W (fp16 hi/lo, resident in TMEM), B = F tile (fp16 hi/lo, SMEM,
//       K-major 128B swizzle), three passes lo*hi + hi*lo + hi*hi: each
//       operand carries 22 significant bits (fp32-level products).  fp16 is
//       used for its 11-bit mantissa; ranges are kept in fp16 by exact
//       power-of-two scaling: x' = x 2^-a (one a per call) and
//       W'_k = W_k 2^-s_k (per component), undone exactly in the epilogue;
//   * per-row log-sum-exp over components: warp max (redux.sync.max.f32),
//     exp2, warp sum (fp32 transpose-reduce over shuffles), combine the 4 warps
//     that share a row, then exchange one (max, sum) pair per row and CTA
//     over distributed shared memory -- no second distance pass;
//   * r = 2^(ll - logZ2); statistics GEMM  T[k, f] += sum_n R^T[k, n] F[n, f]
//       A = R^T (fp16 hi/lo written to TMEM by the epilogue warps),
//       B = the same F tile read MN-major, three passes again;
//     Nk_k = sum r (and, iso, sum r*ll2 for sig) are per-thread sums
//     (thread = component).
//   * per-cluster partials go to the workspace; a second kernel reduces them
//     in a fixed order (deterministic; the reference uses tl.atomic_add).
//
// F enters through a split pass: one read of X writes the fp16 hi/lo feature
// words already in the swizzled per-tile order the MMAs read (plus |x|^2 per
// row for iso), so each stage is filled by one contiguous cp.async.bulk.
//
// Warp roles (640 threads): warps 0-15 epilogue (warp w: lane quadrant w%4,
// row block w/4), warp 16 loads F tiles, warp 17 issues the MMAs, warps 18-19
// are idle.  Every wait is bounded: on timeout the kernel sets an error word
// (outputs become NaN) and leaves its loops.
#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>
#include <climits>
#include <atomic>
#include <mutex>
#include <type_traits>
#include <vector>

#include "fgmm_internal.cuh"
#include "fgmm_ptx.cuh"

namespace fgmm {
namespace {

constexpr int kComps = 128;          // components per CTA (TMEM lanes, MMA M)
constexpr int kMaxDIso = 128;        // largest D of the 128-row isotropic kernel
constexpr int kMaxDIsoWide = 256;    // largest D of the isotropic tensor-core path
constexpr int kMaxDDiag = 96;        // largest D of the stacked diagonal kernel
constexpr int kMaxDDiagWide = 128;   // largest D of the diagonal tensor-core path
constexpr int kEpiWarps = 16;
constexpr int kLoadWarp = kEpiWarps;                        // 16
constexpr int kMmaWarp = kEpiWarps + 1;                     // 17
constexpr int kThreads = (kEpiWarps + 4) * 32;              // 640: 5 warpgroups
constexpr int kMaxCluster = 16;                             // non-portable size, K <= 2048
constexpr int kBlockComps = kComps * 8;                     // components per block (K > 2048)
constexpr int kMaxBlocks = 16;                              // K <= 16384 on the tensor cores
constexpr int kMaxStages = 4;
constexpr int kSplitRows = 4;                               // rows per warp step (split pass)
constexpr int kSms = 148;                                   // B200

// Compile-time shape of one fused-kernel instantiation.
//
// Stage layout (one row tile, fp16 hi/lo feature words, K-major 128B swizzle):
//   iso:  [hi chunk 0 | hi chunk 1 | ... | lo chunk 0 | ...]
//   diag: [hi chunk 0 | lo chunk 0 | hi chunk 1 | lo chunk 1 | ...], so that the
//         hi and lo rows of one 64-feature chunk form a single 128-row B operand:
//         one N=128 MMA gives W_hi F_hi and W_hi F_lo side by side (an N=64 MMA
//         costs as much as an N=128 one), W_lo F_hi is a second, N=64 MMA.
//         W_hi stays in TMEM (A of the N=128 MMA) and W_lo moves to shared
//         memory (A of the N=64 MMA, whose B is half as wide).
//
// The wide kernels (isotropic 128 < D <= 256, diagonal 96 < D <= 128: up to
// 256 features) use 64-row tiles with the iso stage layout, W_hi in TMEM and
// W_lo in shared memory: TMEM T 256 | S 64 | R^T 64 | W_hi 128.
//
// CL is the largest cluster the instantiation runs with: 8 (K <= 1024, and
// the 1024-component blocks of larger K), or 16 for one pass over
// K <= 2048 (the exchange buffer grows; the 128-row kernel drops to 2 stages).
template <int ROWS, bool DIAG, int MAXFEAT, int STAGES, bool WLO_SMEM, bool STACK, int CL = 8>
struct Cfg {
  static constexpr int kCluster = CL;
  static constexpr int kRows = ROWS;                  // rows per tile (distance MMA N)
  static constexpr bool kDiag = DIAG;
  static constexpr bool kStack = STACK;               // [hi | lo] rows per chunk (diag)
  static constexpr bool kWloSmem = WLO_SMEM;          // W_lo in shared memory
  static constexpr int kStages = STAGES;              // F tile buffers
  static constexpr int kMaxFeat = MAXFEAT;
  static constexpr int kMaxD = DIAG ? MAXFEAT / 2 : MAXFEAT;
  static constexpr int kChunk = ROWS * 128;           // bytes of one 64-feature chunk
  static constexpr int kFStride = STACK ? 2 * kChunk : kChunk;  // chunk stride in a stage
  static constexpr int kRB = ROWS / 4;                // rows per epilogue warp (phase A)
  static constexpr int kSCols = STACK ? 2 * ROWS : ROWS;        // stacked: [hh + lh | hl]
  static constexpr int kWCols = WLO_SMEM ? kMaxFeat / 2 : kMaxFeat;  // W hi (+ lo)
  static constexpr int kWSmem = WLO_SMEM ? kComps * 2 * kMaxFeat : 0;  // W lo, bytes
  static constexpr int kNV = (kMaxD + 127) / 128;     // float4 of x per lane (split pass)
  // Distance passes per tile: the wide kernel evaluates S over features
  // [0, 128) and [128, nfeat) separately and adds the halves in fp32
  // registers, so no accumulator chain runs over more than 8 K-steps.
  static constexpr int kHalves = (!STACK && MAXFEAT > 128) ? 2 : 1;
  // TMEM column map (512 columns allocated)
  static constexpr uint32_t kColT = 0;                // statistics accumulator
  static constexpr uint32_t kColS = kMaxFeat;         // distance accumulator
  static constexpr uint32_t kColR = kColS + kSCols;   // R^T hi (ROWS/2) + lo (ROWS/2)
  static constexpr uint32_t kColW = kColR + ROWS;     // W hi (+ W lo when in TMEM)
  static_assert(kColW + kWCols <= 512, "TMEM budget");
  // byte offset of the lo half of a stage
  __host__ __device__ static constexpr int lo_offset(int nch) {
    return STACK ? kChunk : nch * kChunk;
  }
  static_assert(kStages <= kMaxStages, "stage count");
  static_assert(kRB == 16 || kRB == 32, "epilogue row block");
  static constexpr int kGroups = ROWS == 128 ? 4 : 1;  // independent epilogue row groups
};
using IsoCfg = Cfg<128, false, kMaxDIso, 3, false, false>;
using DiagCfg = Cfg<64, true, 2 * kMaxDDiag, 3, true, true>;
using WideCfg = Cfg<64, false, kMaxDIsoWide, 2, true, false>;
using DiagWideCfg = Cfg<64, true, 2 * kMaxDDiagWide, 2, true, false>;
using IsoCfg16 = Cfg<128, false, kMaxDIso, 2, false, false, 16>;
using DiagCfg16 = Cfg<64, true, 2 * kMaxDDiag, 3, true, true, 16>;
using WideCfg16 = Cfg<64, false, kMaxDIsoWide, 2, true, false, 16>;
using DiagWideCfg16 = Cfg<64, true, 2 * kMaxDDiagWide, 2, true, false, 16>;
enum CfgId { kCfgIso = 0, kCfgDiag = 1, kCfgWide = 2, kCfgDiagWide = 3 };
// Calls f with a value of the configuration type (an empty struct); big:
// the 16-CTA-cluster instantiation of the same layout.
template <class F>
decltype(auto) with_cfg(int id, F&& f, bool big = false) {
  if (big) {
    if (id == kCfgDiag) return f(DiagCfg16{});
    if (id == kCfgWide) return f(WideCfg16{});
    if (id == kCfgDiagWide) return f(DiagWideCfg16{});
    return f(IsoCfg16{});
  }
  if (id == kCfgDiag) return f(DiagCfg{});
  if (id == kCfgWide) return f(WideCfg{});
  if (id == kCfgDiagWide) return f(DiagWideCfg{});
  return f(IsoCfg{});
}

struct TcParams {
  const uint8_t* xsplit;     // [num_tiles][stage bytes] swizzled fp16 hi/lo features
  const float* xsq;          // iso: [num_tiles * rows] |x|^2 (0 for padding rows)
  int64_t N;
  int K, D, Dp, nfeat, nch, C;
  int num_tiles;
  const __half* Whi;         // [C*128][nfeat]  W'_k = W_k 2^-s_k
  const __half* Wlo;
  const float4* consts;      // [C*128] {c0', ish (iso), c0 (iso), s_k}
  const int* xscale;         // [0] = max|mu| (or max|mu - c|) bits -> a
  // isotropic: nonzero when the components' variances differ (null: treat
  // them as different); written by tc_prep_kernel
  const int* nonuniform = nullptr;
  // Mode 0 (single pass): logZ[row] out, natural log.  Component blocks of
  // more than 1024 components (K > 1024) run in two phases: mode 1 writes
  // each row's log-sum-exp over this launch's components to logZ[row] in
  // log2 units; mode 2 reads the combined log2 normaliser from logZ[row] and
  // forms r = 2^(ll - lz2) and the statistics without any exchange.
  float* logZ;
  float* part;               // [clusters][C*128][plen]
  int plen;
  int* err;
  // isotropic kernels (modes 0 and 2): (row, component) pairs whose expanded
  // distance may carry more error than logZ's tolerance allows are appended
  // here (null: none) for tc_refine_iso_kernel; mc[k] = |mu_k - c| for this
  // launch's components
  const float* mc = nullptr;
  int4* refine = nullptr;     // {row of the call, component of the call, r bits, ll (log2) bits}
  int* refine_count = nullptr;
  int refine_cap = 0;
  int row_base = 0;           // first row of this launch within the call
  int comp_base = 0;          // first component of this launch within the call
};

struct __align__(8) SmemCtl {
  uint64_t xfull[kMaxStages];
  uint64_t xempty[kMaxStages];
  uint64_t s_full, s_empty, r_full, r_empty, t_done;
  uint64_t xchg_full[2][4];  // [tile parity][row group]
  uint64_t e_bar[2][4];      // epilogue sync points per row group (one arrive per warp)
  uint64_t e_end;
  uint32_t tmem_base;
  volatile int abort_flag;
};

// Bounded wait on a CTA-local (or, kCluster, cluster-scope) mbarrier phase.
template <bool kCluster = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, SmemCtl* ctl, int* err,
                                          int code) {
  return mbar_wait_flag<kCluster>(b, parity, &ctl->abort_flag, err, code);
}

#include "fgmm_tc_iso.cuh"

// ---------------------------------------------------------------------------
// Isotropic prep, one block per component (Kpad blocks of 128 threads), in
// the centred form m = mu - c (c = mean of the mu's, as for diag):
//   ish = 1/2 e^{-lss} log2 e,  c0 = (log pi - D/2 (log 2pi + lss)) log2 e,
//   c0' = c0 - ish |m|^2             (flash_gmm_h100.py:286-291)
//   W = 2 ish m, W' = W 2^-s (s from max|W_k|), split into fp16 hi/lo.
// Components >= K get W = 0, ish = 0, c0' = c0 = -1e30 so they carry zero
// responsibility; -inf log-weights are clamped to the same finite floor.
// ---------------------------------------------------------------------------
// Threads of the isotropic prep block: one per padded feature, 4 or 8 warps.
inline int prep_threads(int Dp) { return Dp > 128 ? 256 : 128; }

__global__ void __launch_bounds__(256) tc_prep_kernel(
    const float* __restrict__ mu, int64_t smk, int64_t smd, const float* __restrict__ lss,
    const float* __restrict__ lpi, const float* __restrict__ cvec, int K, int D, int Dp,
    __half* __restrict__ Whi, __half* __restrict__ Wlo, float4* __restrict__ consts,
    int* __restrict__ nonuniform, float* __restrict__ mc = nullptr) {
  const int k = blockIdx.x;
  const bool valid = k < K;
  if (nonuniform != nullptr && threadIdx.x == 0 && valid && lss[k] != lss[0])
    atomicOr(nonuniform, 1);
  double ish = 0.0, c0 = -1e30;
  if (valid) {
    const double l = (double)lss[k];
    ish = 0.5 * exp(-l) * kLog2E;
    c0 = ((double)lpi[k] - 0.5 * D * (kLog2Pi + l)) * kLog2E;
  }
  const int d = threadIdx.x;  // Dp <= blockDim.x
  const int nw = blockDim.x >> 5;
  double m = 0.0;
  if (valid && d < D) m = (double)mu[(int64_t)k * smk + (int64_t)d * smd] - (double)cvec[d];
  const float w = (float)(2.0 * ish * m);
  __shared__ double s_sq[8];
  __shared__ float s_wmax[8];
  double sq = m * m;
  float wmax = fabsf(w);
  for (int o = 16; o > 0; o >>= 1) {
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
    wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
  }
  if ((threadIdx.x & 31) == 0) {
    s_sq[threadIdx.x >> 5] = sq;
    s_wmax[threadIdx.x >> 5] = wmax;
  }
  __syncthreads();
  double musq = 0.0;
  float wm = 0.f;
  for (int i = 0; i < nw; ++i) {
    musq += s_sq[i];
    wm = fmaxf(wm, s_wmax[i]);
  }
  const int sk = scale_exp(wm);
  if (d < Dp) {
    const float ws = ldexpf(w, -sk);
    const __half h = __float2half_rn(ws);
    Whi[(size_t)k * Dp + d] = h;
    Wlo[(size_t)k * Dp + d] = __float2half_rn(ws - __half2float(h));
  }
  if (threadIdx.x == 0) {
    double c0p = c0 - ish * musq;
    if (!(c0 > -1e30)) { c0 = -1e30; c0p = -1e30; }
    if (c0p < -1e30) c0p = -1e30;
    consts[k] = make_float4((float)c0p, (float)ish, (float)c0, (float)sk);
    if (mc != nullptr) mc[k] = (float)sqrt(musq);
  }
}

// ---------------------------------------------------------------------------
// Diagonal prep, one block per component (Kpad blocks of 128 threads; thread
// d < Dp):  A = 1/2 e^{-lss} log2 e,  B = 2 A (mu - c),
//   c0  = (log pi - 1/2 (D log 2pi + sum_d lss)) log2 e     (diag:335-339)
//   c0' = c0 - sum_d A (mu - c)^2
//   W = [-A 2^{2a}, B 2^a] (features [(x-c)^2 2^-2a, (x-c) 2^-a]), scaled by
//   a per-component power of two and split into fp16 hi/lo.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) tc_prep_diag_kernel(
    const float* __restrict__ mu, int64_t smk, int64_t smd, const float* __restrict__ lss,
    const float* __restrict__ lpi, const float* __restrict__ cvec, const int* __restrict__ amax,
    int K, int D, int Dp, __half* __restrict__ Whi, __half* __restrict__ Wlo,
    float4* __restrict__ consts) {
  const int k = blockIdx.x;
  const bool valid = k < K;
  const int a = x_scale_exp<true>(__int_as_float(*amax));
  const int d = threadIdx.x;
  double A = 0.0, B = 0.0, l = 0.0, am2 = 0.0;
  if (valid && d < D) {
    l = (double)lss[(int64_t)k * D + d];
    const double m = (double)mu[(int64_t)k * smk + (int64_t)d * smd] - (double)cvec[d];
    A = 0.5 * exp(-l) * kLog2E;
    B = 2.0 * A * m;
    am2 = A * m * m;
  }
  const float wa = (float)ldexp(-A, 2 * a), wb = (float)ldexp(B, a);
  __shared__ double s_l[4], s_am2[4];
  __shared__ float s_wmax[4];
  float wmax = fmaxf(fabsf(wa), fabsf(wb));
  for (int o = 16; o > 0; o >>= 1) {
    l += __shfl_xor_sync(0xffffffffu, l, o);
    am2 += __shfl_xor_sync(0xffffffffu, am2, o);
    wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
  }
  if ((threadIdx.x & 31) == 0) {
    s_l[threadIdx.x >> 5] = l;
    s_am2[threadIdx.x >> 5] = am2;
    s_wmax[threadIdx.x >> 5] = wmax;
  }
  __syncthreads();
  const float wm = fmaxf(fmaxf(s_wmax[0], s_wmax[1]), fmaxf(s_wmax[2], s_wmax[3]));
  const int sk = scale_exp(wm);
  if (d < Dp) {
    const int nfeat = 2 * Dp;
    float ws = ldexpf(wa, -sk);
    __half h = __float2half_rn(ws);
    Whi[(size_t)k * nfeat + d] = h;
    Wlo[(size_t)k * nfeat + d] = __float2half_rn(ws - __half2float(h));
    ws = ldexpf(wb, -sk);
    h = __float2half_rn(ws);
    Whi[(size_t)k * nfeat + Dp + d] = h;
    Wlo[(size_t)k * nfeat + Dp + d] = __float2half_rn(ws - __half2float(h));
  }
  if (threadIdx.x == 0) {
    double c0 = -1e30, c0p = -1e30;
    if (valid) {
      const double lsum = s_l[0] + s_l[1] + s_l[2] + s_l[3];
      const double am2s = s_am2[0] + s_am2[1] + s_am2[2] + s_am2[3];
      c0 = ((double)lpi[k] - 0.5 * ((double)D * kLog2Pi + lsum)) * kLog2E;
      c0p = c0 - am2s;
      if (!(c0 > -1e30)) { c0 = -1e30; c0p = -1e30; }
      if (c0p < -1e30) c0p = -1e30;
    }
    consts[k] = make_float4((float)c0p, 0.f, (float)c0, (float)sk);
  }
}

// ---------------------------------------------------------------------------
// The fused kernel.
// ---------------------------------------------------------------------------
template <class G, int MODE>
__global__ void __launch_bounds__(kThreads, 1) tc_fused_kernel(const TcParams p) {
  constexpr int R = G::kRows, RB = G::kRB, NS = G::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int stage_bytes = 2 * p.nch * G::kChunk;    // hi + lo
  uint8_t* xs = smem;                                // [NS][stage]
  uint8_t* whs = smem + NS * stage_bytes;            // diag: W lo, 16 KB per 64 features
  float* xsq = reinterpret_cast<float*>(whs + G::kWSmem);  // iso: [NS][R]
  float* red_m = xsq + NS * R;                       // [16 warps][RB]
  float* red_l = red_m + kEpiWarps * RB;             // [16 warps][RB]
  float* scale_s = red_l + kEpiWarps * RB;           // [R rows] logZ2 (4 R reserved)
  float* fin = scale_s + 4 * R;                      // [8][128] end-of-kernel sums
  constexpr int CL = G::kCluster;
  float2* xchg = reinterpret_cast<float2*>(fin + 8 * kComps);  // [2][CL][R]
  float* lzs = reinterpret_cast<float*>(xchg + 2 * CL * R);    // mode 2: [NS][R]
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(lzs + NS * R);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int cluster_id = blockIdx.x / p.C;
  const int num_clusters = gridDim.x / p.C;
  const int ntiles = (p.num_tiles - cluster_id + num_clusters - 1) / num_clusters;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&ctl->xfull[s], 1);   // loader's arrive.expect_tx + bulk-copy bytes
      mbar_init(&ctl->xempty[s], 1);  // commit of the stats MMA that read the stage
    }
    mbar_init(&ctl->s_full, 1);
    mbar_init(&ctl->s_empty, kEpiWarps);
    mbar_init(&ctl->r_full, kEpiWarps);
    mbar_init(&ctl->r_empty, 1);
    mbar_init(&ctl->t_done, 1);
    for (int gq = 0; gq < G::kGroups; ++gq) {
      mbar_init(&ctl->xchg_full[0][gq], 1);   // local arrive.expect_tx + st.async bytes
      mbar_init(&ctl->xchg_full[1][gq], 1);
      mbar_init(&ctl->e_bar[0][gq], kEpiWarps / G::kGroups);
      mbar_init(&ctl->e_bar[1][gq], kEpiWarps / G::kGroups);
    }
    mbar_init(&ctl->e_end, kEpiWarps);
    ctl->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {  // allocate all 512 TMEM columns (one CTA per SM)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(&ctl->tmem_base))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Components of this thread (epilogue warps): lane quadrant q, row block cb.
  const int q = warp & 3, cb = warp >> 2;
  const int kl = q * 32 + lane;                 // local component (TMEM lane)
  const int kg = (int)rank * kComps + kl;       // global component
  float4 kc = make_float4(-1e30f, 0.f, -1e30f, 0.f);
  if (warp < kEpiWarps) kc = p.consts[kg];
  const int xa = x_scale_exp<G::kDiag>(__int_as_float(*p.xscale));   // x' = x 2^-xa

  for (int i = threadIdx.x; i < NS * stage_bytes / 16; i += kThreads)
    reinterpret_cast<uint4*>(xs)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t wcols = (uint32_t)(p.nfeat / 2);

  // W rows (A operand of the distance GEMM), lane = component: iso hi and lo
  // into TMEM; diag hi into TMEM and lo into shared memory (K-major swizzled).
  if (warp < 4) {
    const uint4* wh = reinterpret_cast<const uint4*>(p.Whi + (size_t)kg * p.nfeat);
    const uint4* wl = reinterpret_cast<const uint4*>(p.Wlo + (size_t)kg * p.nfeat);
    for (int s = 0; s < p.nfeat / 16; ++s) {
      uint32_t v[8];
      uint4 a = wh[2 * s], b = wh[2 * s + 1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      tmem_st8(tmem + ((uint32_t)(q * 32) << 16) + G::kColW + 8 * s, v);
      a = wl[2 * s];
      b = wl[2 * s + 1];
      if constexpr (G::kWloSmem) {
        *reinterpret_cast<uint4*>(whs + xoff(kl, 16 * s, kComps * 128)) = a;
        *reinterpret_cast<uint4*>(whs + xoff(kl, 16 * s + 8, kComps * 128)) = b;
      } else {
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        tmem_st8(tmem + ((uint32_t)(q * 32) << 16) + G::kColW + wcols + 8 * s, v);
      }
    }
    tmem_wait_st();
  }
  if constexpr (G::kWloSmem) fence_async_smem();  // W lo: generic stores -> tensor-core reads
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // peers' barriers are initialised before any remote arrive
  tc_fence_after();

  if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_dist = idesc_f16(R, false);
      const uint32_t id_dist2 = idesc_f16(2 * R, false);  // diag: [F_hi; F_lo] rows
      const uint32_t id_stat = idesc_f16(64 * p.nch, true);
      const int ksd = p.nfeat / 16;
      const uint32_t lo_off = (uint32_t)G::lo_offset(p.nch);
      bool first_stats = true;
      // Descriptors are formed once per stage as their low words and advanced
      // by constant offsets (>> 4), in fully unrolled loops: the issuing lane
      // shares its sub-partition with epilogue warps, and a per-MMA
      // descriptor computation left the tensor pipe idle between MMAs.  A
      // pass over all K-steps is issued straight-line; shorter ones (fewer
      // features) by a plain loop: an unrolled loop with a guard per MMA
      // issued slower than either.
      const uint32_t xs0 = smem_u32(xs), wsm = smem_u32(whs);
      auto issue_stats = [&](int jj) -> void {
        const uint32_t xhi = xs0 + (uint32_t)((jj % NS) * stage_bytes);
        const uint32_t dhi = desc_lo_mnmajor(xhi, G::kFStride);
        const uint32_t dlo = desc_lo_mnmajor(xhi + lo_off, G::kFStride);
        // terms lo*hi, hi*lo, then hi*hi (smallest magnitudes first); K-step s
        // = rows 16s..16s+15, 2048 bytes apart
#pragma unroll
        for (int t = 0; t < 3; ++t) {
          const uint32_t acol = tmem + G::kColR + (t == 0 ? (uint32_t)(R / 2) : 0u);
          const uint32_t bd = t == 1 ? dlo : dhi;
#pragma unroll
          for (int s = 0; s < R / 16; ++s)
            mma_ts2(tmem + G::kColT, acol + 8u * (uint32_t)s, bd + (uint32_t)(s * (2048 >> 4)),
                    kDescHi, id_stat, (first_stats && t == 0 && s == 0) ? 0u : 1u);
        }
        first_stats = false;
        tc_commit(&ctl->r_empty);
        tc_commit(&ctl->xempty[jj % NS]);
      };
      constexpr int H = G::kHalves;
      bool ok = true;
      for (int j = 0; j < ntiles && ok; ++j) {
        const int b = j % NS;
        if (!mbar_wait(&ctl->xfull[b], (j / NS) & 1, ctl, p.err, 1)) break;
        const uint32_t xhi = xs0 + (uint32_t)(b * stage_bytes);
        const uint32_t dhi = desc_lo_kmajor(xhi), dlo = desc_lo_kmajor(xhi + lo_off);
        const uint32_t dw = desc_lo_kmajor(wsm);
        if constexpr (G::kStack) {
          if (j >= 1 && !mbar_wait(&ctl->s_empty, (j - 1) & 1, ctl, p.err, 2)) break;
          tc_fence_after();
          // per K-step: W_hi [F_hi; F_lo] (N = 2R: columns [hh | hl]), then
          // W_lo F_hi (N = R) into the hh columns
          auto stack_mma = [&](int s) {
            const uint32_t fd = dhi + (uint32_t)(((s >> 2) * G::kFStride + (s & 3) * 32) >> 4);
            const uint32_t wd = dw + (uint32_t)(((s >> 2) * (kComps * 128) + (s & 3) * 32) >> 4);
            mma_ts2(tmem + G::kColS, tmem + G::kColW + 8u * (uint32_t)s, fd, kDescHi, id_dist2,
                    s == 0 ? 0u : 1u);
            mma_ss2(tmem + G::kColS, wd, fd, kDescHi, id_dist, 1u);
          };
          if (ksd == G::kMaxFeat / 16) {  // all features: straight-line issue
#pragma unroll
            for (int s = 0; s < G::kMaxFeat / 16; ++s) stack_mma(s);
          } else {
            for (int s = 0; s < ksd; ++s) stack_mma(s);
          }
          tc_commit(&ctl->s_full);
        } else {
          // terms W_lo x_hi, W_hi x_lo, W_hi x_hi (smallest magnitudes first),
          // per pass h over K-steps [8h, 8h + 8); W_lo from shared memory in
          // the wide kernel.  Pass (j, h) is s_full / s_empty phase j H + h.
          constexpr int kKS = H == 1 ? G::kMaxFeat / 16 : 8;  // K-steps per pass, at most
          static_assert(kKS <= 8, "distance pass length");
          for (int h = 0; h < H; ++h) {
            const int ph = j * H + h;
            if (ph >= 1 && !mbar_wait(&ctl->s_empty, (ph - 1) & 1, ctl, p.err, 2)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const int s0 = 8 * h;
            const int ns = ksd - s0 < kKS ? ksd - s0 : kKS;
            auto dist_mma = [&](int t, int s, uint32_t acc) {
              const uint32_t bd = t == 1 ? dlo : dhi;
              const uint32_t off = (uint32_t)(((s >> 2) * G::kChunk + (s & 3) * 32) >> 4);
              if (G::kWloSmem && t == 0)
                mma_ss2(tmem + G::kColS,
                        dw + (uint32_t)(((s >> 2) * (kComps * 128) + (s & 3) * 32) >> 4),
                        bd + off, kDescHi, id_dist, acc);
              else
                mma_ts2(tmem + G::kColS, tmem + G::kColW + (t == 0 ? wcols : 0u) + 8u * (uint32_t)s,
                        bd + off, kDescHi, id_dist, acc);
            };
            if (ns == kKS) {  // a full pass: straight-line issue
#pragma unroll
              for (int t = 0; t < 3; ++t)
#pragma unroll
                for (int i = 0; i < kKS; ++i) dist_mma(t, s0 + i, (t == 0 && i == 0) ? 0u : 1u);
            } else {
              for (int t = 0; t < 3; ++t)
                for (int i = 0; i < ns; ++i) dist_mma(t, s0 + i, (t == 0 && i == 0) ? 0u : 1u);
            }
            tc_commit(&ctl->s_full);
          }
          if (!ok) break;
        }
        if (MODE == 1) {
          // LSE only: the stage is free once the epilogue has read this
          // tile's distances and |x|^2 words (its last s_empty arrival)
          if (!mbar_wait(&ctl->s_empty, (j * H + H - 1) & 1, ctl, p.err, 2)) break;
          mbar_arrive(&ctl->xempty[b]);
          continue;
        }
        if (j >= 1) {
          if (!mbar_wait(&ctl->r_full, (j - 1) & 1, ctl, p.err, 4)) break;
          tc_fence_after();
          issue_stats(j - 1);
        }
      }
      if (MODE != 1 && ntiles >= 1 && !ctl->abort_flag) {
        if (mbar_wait(&ctl->r_full, (ntiles - 1) & 1, ctl, p.err, 4)) {
          tc_fence_after();
          issue_stats(ntiles - 1);
          tc_commit(&ctl->t_done);
        }
      }
    }
    __syncwarp();
  } else if (warp == kLoadWarp) {
    // ------------------------------------------------------------ F loader
    if (lane == 0) {
      const uint32_t tx = (uint32_t)stage_bytes + (G::kDiag ? 0u : (uint32_t)R * 4u) +
                          (MODE == 2 ? (uint32_t)R * 4u : 0u);
      for (int j = 0; j < ntiles; ++j) {
        const int b = j % NS;
        const int64_t tile = cluster_id + (int64_t)j * num_clusters;
        if (!mbar_wait(&ctl->xempty[b], ((j / NS) & 1) ^ 1, ctl, p.err, 8)) break;
        mbar_arrive_expect_tx(&ctl->xfull[b], tx);
        bulk_g2s(smem_u32(xs + b * stage_bytes), p.xsplit + tile * stage_bytes,
                 (uint32_t)stage_bytes, &ctl->xfull[b]);
        if (!G::kDiag)
          bulk_g2s(smem_u32(xsq + b * R), p.xsq + tile * R, (uint32_t)R * 4u, &ctl->xfull[b]);
        if (MODE == 2)
          bulk_g2s(smem_u32(lzs + b * R), p.logZ + tile * R, (uint32_t)R * 4u, &ctl->xfull[b]);
      }
    }
    __syncwarp();
  } else if (warp < kEpiWarps) {
    // ------------------------------------------------------------- epilogue
    // Per tile: A) S^T -> ll, warp max / exp2 / warp sum per row;
    // B) combine the 4 lane quadrants per row and send one (max, sum) pair to
    // every CTA of the cluster; C) combine the cluster's pairs -> logZ2
    // per row; D) r = 2^(ll - logZ2), per-component sums, R^T
    // (fp16 hi/lo) into TMEM for the statistics GEMM.
    const float c0p = kc.x, ish = kc.y, c0 = kc.z;
    const float sck = ldexpf(1.0f, (G::kDiag ? 0 : xa) + (int)kc.w);  // S = S' 2^(a + s_k)
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float nk_acc = 0.f, rll_acc = 0.f;
    // Isotropic logZ refinement gate: the expanded distance's error grows
    // with ish |x - c| |mu_k - c|; pairs with r >= 2^-8 where 64 x 2^-23 of
    // that exceeds logZ's tolerance are listed for tc_refine_iso_kernel (64
    // units: these kernels sum up to 16 K-steps, in two chains on the wide
    // one).  gate2() = (64 x 2^-23 ish |mu_k - c|)^2, formed where it is used
    // from |mu_k - c| loaded once (a load per tile would sit on the
    // epilogue's latency chain).
    const float mck = (!G::kDiag && p.refine != nullptr && warp < kEpiWarps) ? p.mc[kg] : 0.f;
    auto gate2 = [&]() -> float {
      const float rbk = ish * mck * 7.62939453125e-06f;
      return rbk * rbk;
    };
    const int tid_e = threadIdx.x;                 // 0..511
    const int g = lane >> 3;                       // lane group for row work
    const bool row_owner = 8 * warp < R;           // warps that own rows in B / C
    // Row groups: with 128-row tiles the 4 warps of row block cb own its 32
    // rows end to end (A, B/C and D), so each block synchronises and
    // exchanges on its own and the blocks drift out of phase; 64-row tiles
    // use one group.
    const int grp = G::kGroups == 4 ? cb : 0;
    constexpr int kGroupRows = R / G::kGroups;
    const int Rw = 8 * warp + (lane & 7);          // row owned in B / C
    for (int t = 0; t < ntiles; ++t) {
      const int b = t % NS;
      const int64_t row0 = (int64_t)(cluster_id + (int64_t)t * num_clusters) * R;
      // ---- A
      constexpr int H = G::kHalves;
      if (!mbar_wait(&ctl->s_full, (t * H) & 1, ctl, p.err, 16)) break;
      if (!mbar_wait(&ctl->xfull[b], (t / NS) & 1, ctl, p.err, 4096)) break;
      tc_fence_after();
      float ll[RB], pv[RB];
      {
        uint32_t sv[RB];
        if constexpr (H == 2) {
          // first distance pass into registers, then the second one added
          tmem_ld16(tmem + lane_base + G::kColS + RB * cb, sv);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctl->s_empty);
          if (!mbar_wait(&ctl->s_full, (t * H + 1) & 1, ctl, p.err, 16)) break;
          tc_fence_after();
          uint32_t s2[RB];
          tmem_ld16(tmem + lane_base + G::kColS + RB * cb, s2);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < RB; ++i)
            sv[i] = __float_as_uint(__uint_as_float(sv[i]) + __uint_as_float(s2[i]));
        } else if constexpr (RB == 32) {
          tmem_ld32(tmem + lane_base + G::kColS + RB * cb, sv);
          tmem_wait_ld();
        } else if constexpr (G::kStack) {
          uint32_t sl[RB];  // the W_hi F_lo columns
          tmem_ld16(tmem + lane_base + G::kColS + RB * cb, sv);
          tmem_ld16(tmem + lane_base + G::kColS + R + RB * cb, sl);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < RB; ++i)
            sv[i] = __float_as_uint(__uint_as_float(sv[i]) + __uint_as_float(sl[i]));
        } else {
          tmem_ld16(tmem + lane_base + G::kColS + RB * cb, sv);
          tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (MODE != 1 && lane == 0) mbar_arrive(&ctl->s_empty);
        if constexpr (G::kDiag) {
#pragma unroll
          for (int i = 0; i < RB; ++i) ll[i] = fmaf(__uint_as_float(sv[i]), sck, c0p);
        } else {
          const float* xq = xsq + b * R + RB * cb;
#pragma unroll
          for (int i = 0; i < RB; i += 4) {
            const float4 s4 = *reinterpret_cast<const float4*>(xq + i);
            ll[i + 0] = fmaf(__uint_as_float(sv[i + 0]), sck, fmaf(-ish, s4.x, c0p));
            ll[i + 1] = fmaf(__uint_as_float(sv[i + 1]), sck, fmaf(-ish, s4.y, c0p));
            ll[i + 2] = fmaf(__uint_as_float(sv[i + 2]), sck, fmaf(-ish, s4.z, c0p));
            ll[i + 3] = fmaf(__uint_as_float(sv[i + 3]), sck, fmaf(-ish, s4.w, c0p));
          }
        }
      }
      if (MODE == 1) {  // distances and |x|^2 read: the MMA warp frees the stage
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->s_empty);
      }
      if constexpr (MODE == 2) {
        // known log-normaliser: r = 2^(ll - lz2) directly (rows past N give 0)
        const float* lzr = lzs + b * R + RB * cb;
#pragma unroll
        for (int i = 0; i < RB; ++i)
          pv[i] = (row0 + RB * cb + i < p.N) ? ex2(ll[i] - lzr[i]) : 0.f;
      } else {
      // Row maxima over this warp's 32 components (uniform across lanes),
      // p = 2^(ll - m), then the row sums by a transpose-reduce: log2(32)
      // shuffle rounds, each halving the rows a lane carries, leave the sum
      // of row r in lane r (RB = 16: lane r & 15).  Deterministic fp32 order.
      // The first round is fused with the exponentials to keep registers low.
      {
        constexpr int H = RB / 2;
        float sv[H];
#pragma unroll
        for (int i = 0; i < H; ++i) {
          const float ma = redux_max(ll[i]), mb = redux_max(ll[i + H]);
          pv[i] = ex2(ll[i] - ma);
          pv[i + H] = ex2(ll[i + H] - mb);
          if (lane == 0) {
            red_m[warp * RB + i] = ma;
            red_m[warp * RB + i + H] = mb;
          }
          if constexpr (RB == 32) {
            const bool upper = (lane & 16) != 0;
            const float send = upper ? pv[i] : pv[i + H];
            const float keep = upper ? pv[i + H] : pv[i];
            sv[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
          } else {
            // 16 rows on 32 lanes: fold lanes l and l^16 first, then halve
            float u = pv[i] + __shfl_xor_sync(0xffffffffu, pv[i], 16);
            float w = pv[i + H] + __shfl_xor_sync(0xffffffffu, pv[i + H], 16);
            const bool upper = (lane & 8) != 0;
            sv[i] = (upper ? w : u) + __shfl_xor_sync(0xffffffffu, upper ? u : w, 8);
          }
        }
#pragma unroll
        for (int half = H / 2; half >= 1; half >>= 1) {  // lane bit of the round = half
          const bool upper = (lane & half) != 0;
#pragma unroll
          for (int i = 0; i < half; ++i) {
            const float send = upper ? sv[i] : sv[i + half];
            const float keep = upper ? sv[i + half] : sv[i];
            sv[i] = keep + __shfl_xor_sync(0xffffffffu, send, half);
          }
        }
        if (lane < RB) red_l[warp * RB + lane] = sv[0];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->e_bar[0][grp]);
      if (!mbar_wait(&ctl->e_bar[0][grp], t & 1, ctl, p.err, 256)) break;

      // ---- B + C: warp w < R/8 owns rows Rw = 8w + (lane & 7); lane group g
      // handles lane quadrant g and cluster peers g + 4 j (j < CL / 4).
      const int slot = t & 1;
      if (row_owner) {
        const int ri = Rw % RB, blk = Rw / RB;
        const float mg = red_m[(g + 4 * blk) * RB + ri];
        const float ug = red_l[(g + 4 * blk) * RB + ri];
        float M = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, 8));
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 16));
        float L = ug * ex2(mg - M);
        L += __shfl_xor_sync(0xffffffffu, L, 8);
        L += __shfl_xor_sync(0xffffffffu, L, 16);
        const uint32_t my_slot = smem_u32(&xchg[(slot * CL + rank) * R + Rw]);
        const int rg = Rw / kGroupRows;               // row group of this row (== grp)
        const uint32_t my_bar = smem_u32(&ctl->xchg_full[slot][rg]);
        if (tid_e == 32 * (rg * kGroupRows / 8))      // first owner warp of the group, lane 0
          mbar_arrive_expect_tx(&ctl->xchg_full[slot][rg], (uint32_t)(p.C * kGroupRows * 8));
#pragma unroll
        for (int j = 0; j < CL / 4; ++j)
          if (g + 4 * j < p.C)
            st_async_f2(map_to_cta(my_slot, g + 4 * j), M, L, map_to_cta(my_bar, g + 4 * j));
        const bool ok = mbar_wait<true>(&ctl->xchg_full[slot][rg], (t >> 1) & 1, ctl, p.err, 32);
        float2 e[CL / 4];
#pragma unroll
        for (int j = 0; j < CL / 4; ++j) {
          e[j] = make_float2(-3e38f, 0.f);
          if (g + 4 * j < p.C) e[j] = xchg[(slot * CL + g + 4 * j) * R + Rw];
        }
        float GM = e[0].x;
#pragma unroll
        for (int j = 1; j < CL / 4; ++j) GM = fmaxf(GM, e[j].x);
        GM = fmaxf(GM, __shfl_xor_sync(0xffffffffu, GM, 8));
        GM = fmaxf(GM, __shfl_xor_sync(0xffffffffu, GM, 16));
        float GL = e[0].y * ex2(e[0].x - GM);
#pragma unroll
        for (int j = 1; j < CL / 4; ++j) GL += e[j].y * ex2(e[j].x - GM);
        GL += __shfl_xor_sync(0xffffffffu, GL, 8);
        GL += __shfl_xor_sync(0xffffffffu, GL, 16);
        const float lz2 = GM + lg2(GL);
        const bool valid = ok && (row0 + Rw < p.N);
        if (valid && rank == 0 && g == 0) {
          if constexpr (MODE == 1) p.logZ[row0 + Rw] = lz2;
          else p.logZ[row0 + Rw] = lz2 * 0.6931471805599453f;
        }
        if (g == 0) scale_s[Rw] = valid ? lz2 : __int_as_float(0x7f800000);  // +inf: r = 0
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->e_bar[1][grp]);
      if (!mbar_wait(&ctl->e_bar[1][grp], t & 1, ctl, p.err, 512)) break;
      if constexpr (MODE == 1) continue;  // LSE only: no statistics
      }

      // ---- D: r = 2^(ll - logZ2), per-component sums, R^T into TMEM (16 rows at a time)
      const float* sc = scale_s + RB * cb;            // log2 normaliser per row
      float nk_t = 0.f, rll_t = 0.f;
      if constexpr (!G::kDiag) {
        if (p.refine != nullptr) {
          // Rows whose pairs may need the logZ refinement: |x - c|^2 times the
          // warp's largest gate exceeds the row's tolerance (a warp-uniform
          // mask; on most data empty).  For those rows each component forms
          // r = 2^(ll - logZ2) (ll by a select chain, which keeps ll[] in
          // registers) and lists the pair if r >= 2^-8 and its own gate
          // passes.  Done before the R^T words are released, while the
          // stage's |x|^2 and normaliser words are valid.
          const float rb2 = gate2();
          const float rbk2max = redux_max(rb2);
          bool pass = false;
          if (lane < RB) {
            const int ro = RB * cb + lane;
            const float lzv = MODE == 2 ? lzs[b * R + ro] : sc[lane];
            const float tt = 1e-5f * fmaxf(1.44269504f, fabsf(lzv));
            pass = row0 + ro < p.N && xsq[b * R + ro] * rbk2max > tt * tt;
          }
          for (uint32_t m = __ballot_sync(0xffffffffu, pass); m != 0u; m &= m - 1u) {
            const int i = __ffs(m) - 1;
            float lli = ll[0];
#pragma unroll
            for (int jj = 1; jj < RB; ++jj) lli = jj == i ? ll[jj] : lli;
            const int ro = RB * cb + i;  // row within the tile
            const float lzv = MODE == 2 ? lzs[b * R + ro] : sc[i];
            const float tt = 1e-5f * fmaxf(1.44269504f, fabsf(lzv));
            const float r = ex2(lli - lzv);
            if (r >= 0.00390625f && xsq[b * R + ro] * rb2 > tt * tt) {
              const int at = atomicAdd(p.refine_count, 1);
              if (at < p.refine_cap)
                p.refine[at] = make_int4(p.row_base + (int)(row0 + ro), p.comp_base + kg,
                                         __float_as_int(r), __float_as_int(lli));
            }
          }
        }
      }
      if (t >= 1 && !mbar_wait(&ctl->r_empty, (t - 1) & 1, ctl, p.err, 64)) break;
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < RB / 16; ++h) {
        uint32_t rh[8], rl[8];
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const int o = 16 * h + i;
          float r0, r1, r2, r3;
          if constexpr (MODE == 2) {
            r0 = pv[o + 0]; r1 = pv[o + 1]; r2 = pv[o + 2]; r3 = pv[o + 3];
          } else {
            // r = 2^(ll - logZ2) from the distances kept in registers: p of
            // phase A is dead after the row sums, which keeps the epilogue
            // within its 96 registers (no spills) for one more exp2 per pair
            const float4 z4 = *reinterpret_cast<const float4*>(sc + 16 * h + i);
            r0 = ex2(ll[o + 0] - z4.x); r1 = ex2(ll[o + 1] - z4.y);
            r2 = ex2(ll[o + 2] - z4.z); r3 = ex2(ll[o + 3] - z4.w);
          }
          nk_t += (r0 + r1) + (r2 + r3);
          if constexpr (!G::kDiag) {
            rll_t = fmaf(r0, ll[o + 0], rll_t);
            rll_t = fmaf(r1, ll[o + 1], rll_t);
            rll_t = fmaf(r2, ll[o + 2], rll_t);
            rll_t = fmaf(r3, ll[o + 3], rll_t);
          }
          split2(r0, r1, rh[i / 2], rl[i / 2]);
          split2(r2, r3, rh[i / 2 + 1], rl[i / 2 + 1]);
        }
        tmem_st8(tmem + lane_base + G::kColR + (RB / 2) * cb + 8 * h, rh);
        tmem_st8(tmem + lane_base + G::kColR + R / 2 + (RB / 2) * cb + 8 * h, rl);
      }
      nk_acc += nk_t;
      rll_acc += rll_t;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->r_full);
    }

    // End: statistics accumulator -> per-cluster partials.
    fin[cb * kComps + kl] = nk_acc;
    fin[(4 + cb) * kComps + kl] = rll_acc;
    __syncwarp();
    if (lane == 0) mbar_arrive(&ctl->e_end);
    const bool ok = !ctl->abort_flag && ntiles >= 1 &&
                    mbar_wait(&ctl->e_end, 0, ctl, p.err, 1024) && MODE != 1 &&
                    mbar_wait(&ctl->t_done, 0, ctl, p.err, 128);
    float* out = p.part + ((size_t)cluster_id * p.C * kComps + kg) * p.plen;
    if (ok) {
      tc_fence_after();
      for (int blk = cb; 32 * blk < 64 * p.nch; blk += 4) {
        uint32_t tv[32];
        tmem_ld32(tmem + lane_base + G::kColT + 32 * blk, tv);
        tmem_wait_ld();
        for (int i = 0; i < 32; ++i) {
          const int f = 32 * blk + i;
          const float v = __uint_as_float(tv[i]);
          if constexpr (G::kDiag) {
            // partial row {Nk, sum r (x-c) [D], sum r (x-c)^2 [D]}
            if (f < p.Dp) {
              if (f < p.D) out[1 + p.D + f] = ldexpf(v, 2 * xa);
            } else if (f - p.Dp < p.D) {
              out[1 + (f - p.Dp)] = ldexpf(v, xa);
            }
          } else {
            if (f < p.D) out[2 + f] = ldexpf(v, xa);  // T = T' 2^a
          }
        }
      }
      if (cb == 0) {
        const float nk = fin[kl] + fin[kComps + kl] + fin[2 * kComps + kl] + fin[3 * kComps + kl];
        out[0] = nk;
        if constexpr (!G::kDiag) {
          const float rl = fin[4 * kComps + kl] + fin[5 * kComps + kl] + fin[6 * kComps + kl] +
                           fin[7 * kComps + kl];
          out[1] = ish > 0.f ? (c0 * nk - rl) / ish : 0.f;
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
  cluster_sync_all();
}

// ---------------------------------------------------------------------------
// Split pass: X (any strides) -> fp16 hi/lo feature words in the swizzled
// per-tile order of the fused kernel's stage buffers.  One warp per row; lane
// l carries features 4l..4l+3 of x.  Rows past N and features past D are
// zero.  v = hi + lo + O(2^-22 |v|).
//   iso:  features (x-c) 2^-a, plus |x-c|^2 per row;
//   diag: features [((x-c) 2^-a)^2 | (x-c) 2^-a].
// ---------------------------------------------------------------------------
template <class G, class TX>
__global__ void __launch_bounds__(256) tc_split_kernel(
    const TX* __restrict__ X, int64_t sxn, int64_t sxd, int vec_ok, int64_t N, int D, int Dp,
    int nch, int64_t rows_pad, const int* __restrict__ amax, const float* __restrict__ cvec,
    uint8_t* __restrict__ xsplit, float* __restrict__ xsq, int* __restrict__ err,
    unsigned long long* __restrict__ corr = nullptr) {
  constexpr int ROWS = G::kRows, NV = G::kNV;
  constexpr bool DIAG = G::kDiag;
  constexpr int kChunk = ROWS * 128;
  // stage layout: [hi chunks | lo chunks], or [hi | lo] per chunk when stacked
  constexpr int kFS = G::kFStride;
  const int64_t lo = G::lo_offset(nch);
  const int lane = threadIdx.x & 31;
  const int a = x_scale_exp<DIAG>(__int_as_float(*amax));
  const int64_t stage_bytes = (int64_t)2 * nch * kChunk;
  float4 cc[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int f = 128 * v + 4 * lane;
    cc[v] = f < Dp ? *reinterpret_cast<const float4*>(cvec + f) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // Each warp takes kSplitRows consecutive rows per step and issues all of
  // their loads before converting, to keep enough bytes in flight for HBM.
  for (int64_t row0 = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * kSplitRows; row0 < rows_pad;
       row0 += (int64_t)gridDim.x * 8 * kSplitRows) {
    float4 xr[kSplitRows][NV];
#pragma unroll
    for (int u = 0; u < kSplitRows; ++u) {
      const int64_t row = row0 + u;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const int f = 128 * v + 4 * lane;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (f < Dp && row < N) {
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
        xr[u][v] = x;
      }
    }
    // all loads issued: centre and convert (padding features have x = c = 0;
    // rows past N stay 0)
#pragma unroll
    for (int u = 0; u < kSplitRows; ++u) {
      const int64_t row = row0 + u;
      if (row >= rows_pad) break;
      uint8_t* tile = xsplit + (row / ROWS) * stage_bytes;
      const int r = (int)(row % ROWS);
      float sq = 0.f;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const int f = 128 * v + 4 * lane;
        float4 x = xr[u][v];
        if (row < N) {
          x.x -= cc[v].x;
          x.y -= cc[v].y;
          x.z -= cc[v].z;
          x.w -= cc[v].w;
        }
        if (f < Dp) {
          const float4 xs = make_float4(ldexpf(x.x, -a), ldexpf(x.y, -a), ldexpf(x.z, -a),
                                        ldexpf(x.w, -a));
          float mx = fmaxf(fmaxf(fabsf(xs.x), fabsf(xs.y)), fmaxf(fabsf(xs.z), fabsf(xs.w)));
          if (DIAG) mx = fmaxf(mx, mx * mx);
          if (!(mx < 65504.f)) atomicOr(err, 0x10000);  // outside fp16 range (or NaN)
          uint32_t h0, l0, h1, l1;
          split2(xs.x, xs.y, h0, l0);
          split2(xs.z, xs.w, h1, l1);
          const uint32_t off = xoff(r, DIAG ? Dp + f : f, kFS);
          *reinterpret_cast<uint2*>(tile + off) = make_uint2(h0, h1);
          *reinterpret_cast<uint2*>(tile + lo + off) = make_uint2(l0, l1);
          if (DIAG) {
            split2(xs.x * xs.x, xs.y * xs.y, h0, l0);
            split2(xs.z * xs.z, xs.w * xs.w, h1, l1);
            const uint32_t off2 = xoff(r, f, kFS);
            *reinterpret_cast<uint2*>(tile + off2) = make_uint2(h0, h1);
            *reinterpret_cast<uint2*>(tile + lo + off2) = make_uint2(l0, l1);
          }
        }
        if (!DIAG) {
          sq = fmaf(x.x, x.x, sq);
          sq = fmaf(x.y, x.y, sq);
          sq = fmaf(x.z, x.z, sq);
          sq = fmaf(x.w, x.w, sq);
        }
      }
      if (!DIAG) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) {
          xsq[row] = sq;
          if (corr != nullptr && row < N) corr[row] = 0ull;  // logZ refinement sums start at 0
        }
      }
    }
  }
}

// Chunked calls: partial slots [0, n) summed element-wise, in slot order, into
// slot n - 1 (slot_elems floats per slot), while the last chunk's fused kernel
// runs.  The reduction then starts from slot n - 1: the same fp32 summation
// order as summing all slots in one pass.
__global__ void __launch_bounds__(256) tc_part_presum_kernel(float* __restrict__ part, int n,
                                                             int64_t slot_elems) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < slot_elems;
       e += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
#pragma unroll 8
    for (int c = 0; c < n; ++c) s += part[(size_t)c * slot_elems + e];
    part[(size_t)(n - 1) * slot_elems + e] = s;
  }
}

// Isotropic: sum the per-cluster partials {Nk, sig, sum r (x-c)} in cluster
// order; mu_acc = sum r (x-c) + c Nk.  One block per component (thread j sums
// partial column j < D + 2 <= blockDim.x); NaN on a device error.
inline int reduce_threads(int D) { return D + 2 > 256 ? 288 : 256; }

__global__ void __launch_bounds__(288) tc_reduce_kernel(
    const float* __restrict__ part, int clusters, int Kpad, int K, int D,
    const float* __restrict__ cvec, const int* __restrict__ err, float* __restrict__ Nk,
    float* __restrict__ mu_acc, float* __restrict__ sig, int accumulate) {
  const int plen = D + 2, j = threadIdx.x;
  const bool bad = *err != 0;
  __shared__ float s_n;
  for (int k = blockIdx.x; k < K; k += gridDim.x) {
    float s = 0.f;
    if (j < plen) {
#pragma unroll 16
      for (int c = 0; c < clusters; ++c) s += part[((size_t)c * Kpad + k) * plen + j];
    }
    if (j == 0) s_n = s;
    __syncthreads();
    if (j >= 2 && j < plen) s = fmaf(cvec[j - 2], s_n, s);
    __syncthreads();  // s_n is rewritten by the next component
    if (j < plen) {
      if (bad) s = __int_as_float(0x7fc00000);
      float* dst = j == 0 ? &Nk[k] : j == 1 ? &sig[k] : &mu_acc[(size_t)k * D + (j - 2)];
      *dst = accumulate ? *dst + s : s;
    }
  }
}

// Diagonal: sum the partials {Nk, sum r (x-c), sum r (x-c)^2} in cluster
// order, then mu_acc = Tx + c Nk and sig = Txx - 2 m Tx + m^2 Nk with
// m = mu - c (the centred form of diag:258-260).  NaN on a device error.
__global__ void tc_reduce_diag_kernel(const float* __restrict__ part, int clusters, int Kpad,
                                      int K, int D, const float* __restrict__ cvec,
                                      const float* __restrict__ mu, int64_t smk, int64_t smd,
                                      const int* __restrict__ err, float* __restrict__ Nk,
                                      float* __restrict__ mu_acc, float* __restrict__ sig,
                                      int accumulate) {
  const int plen = 1 + 2 * D;
  const bool bad = *err != 0;
  const float qnan = __int_as_float(0x7fc00000);
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < (int64_t)K * (D + 1);
       e += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(e / (D + 1)), j = (int)(e % (D + 1));
    double n = 0.0;
#pragma unroll 16
    for (int c = 0; c < clusters; ++c) n += part[((size_t)c * Kpad + k) * plen];
    if (j == 0) {
      const float v = bad ? qnan : (float)n;
      Nk[k] = accumulate ? Nk[k] + v : v;
      continue;
    }
    const int d = j - 1;
    double tx = 0.0, txx = 0.0;
#pragma unroll 8
    for (int c = 0; c < clusters; ++c) {
      const float* pr = part + ((size_t)c * Kpad + k) * plen;
      tx += pr[1 + d];
      txx += pr[1 + D + d];
    }
    const double cd = cvec[d];
    const double m = (double)mu[(int64_t)k * smk + (int64_t)d * smd] - cd;
    float vm = (float)(tx + cd * n);
    float vs = (float)(txx - 2.0 * m * tx + m * m * n);
    if (bad) vm = vs = qnan;
    const size_t o = (size_t)k * D + d;
    mu_acc[o] = accumulate ? mu_acc[o] + vm : vm;
    sig[o] = accumulate ? sig[o] + vs : vs;
  }
}

// K > 1024: logZ of each row from the per-block log-sum-exps (log2 units),
// lz2 = log2 sum_b 2^lse_b, written in log2 units for phase 2 and in natural
// log for the caller (rows < N).
__global__ void tc_lse_combine_kernel(const float* __restrict__ lse_part, int nb, int64_t npad,
                                      int64_t N, float* __restrict__ lz2,
                                      float* __restrict__ logZ) {
  for (int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; n < N;
       n += (int64_t)gridDim.x * blockDim.x) {
    float m = -3.0e38f;
    for (int b = 0; b < nb; ++b) m = fmaxf(m, lse_part[(size_t)b * npad + n]);
    float sum = 0.f;
    for (int b = 0; b < nb; ++b) sum += ex2(lse_part[(size_t)b * npad + n] - m);
    const float v = m + lg2(sum);
    lz2[n] = v;
    logZ[n] = v * 0.6931471805599453f;
  }
}

// Exact refinement of logZ for the (row, component) pairs listed by the
// isotropic kernels (tc_iso_kernel, and tc_fused_kernel's isotropic
// configurations in modes 0 and 2; log2 units): one warp per pair forms
// |x - mu_k|^2 from the inputs with exact differences (lanes over features,
// a fixed shuffle order), ll = c0_k - ish_k |x - mu_k|^2, and adds
// r (2^(ll - ll_used) - 1) -- the relative change of the row's sum of
// 2^ll -- to corr[row] as a 2^-40 fixed-point integer (integer adds: the
// result does not depend on the order of the pairs).
constexpr double kCorrScale = 1099511627776.0;  // 2^40
template <class TX>
__global__ void __launch_bounds__(256) tc_refine_iso_kernel(
    const int4* __restrict__ pairs, const int* __restrict__ count, int cap,
    const TX* __restrict__ X, int64_t sxn, int64_t sxd, const float* __restrict__ mu,
    int64_t smk, int64_t smd, int D, const float4* __restrict__ consts,
    unsigned long long* __restrict__ corr) {
  const int n = min(*count, cap);
  const int lane = threadIdx.x & 31;
  for (int e = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; e < n;
       e += (gridDim.x * blockDim.x) >> 5) {
    const int4 en = pairs[e];
    const int64_t row = en.x;
    const int k = en.y;
    float d2 = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float diff = ldx(X + row * sxn + (int64_t)d * sxd) - __ldg(mu + (int64_t)k * smk +
                                                                         (int64_t)d * smd);
      d2 = fmaf(diff, diff, d2);
    }
    for (int o = 16; o > 0; o >>= 1) d2 += __shfl_xor_sync(0xffffffffu, d2, o);
    if (lane == 0) {
      const float4 kc = consts[k];  // {c0', ish, c0, s_k}
      const float delta = fmaf(-kc.y, d2, kc.z) - __int_as_float(en.w);
      const double v = (double)__int_as_float(en.z) * ((double)exp2f(delta) - 1.0);
      atomicAdd(corr + row, (unsigned long long)__double2ll_rn(v * kCorrScale));
    }
  }
}

// logZ += ln(1 + corr 2^-40) for the rows of the listed pairs: the first
// pair of a row to take its sum (atomicExch to 0) applies it, once.
__global__ void __launch_bounds__(256) tc_apply_refine_kernel(
    const int4* __restrict__ pairs, const int* __restrict__ count, int cap,
    unsigned long long* __restrict__ corr, float* __restrict__ logZ) {
  const int n = min(*count, cap);
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
    const int row = pairs[e].x;
    const long long v = (long long)atomicExch(corr + row, 0ull);
    if (v != 0) logZ[row] += (float)log1p((double)v / kCorrScale);
  }
}

struct TcPlan {
  bool diag;
  bool iso = false;  // isotropic, K <= 1024, D <= 128: tc_iso_kernel
  int cfg, rows, C, Kpad, Dp, nfeat, nch, num_tiles, clusters, plen;
  bool big;  // 16-CTA clusters (one pass over 1024 < K <= 2048)
  size_t stage_bytes, smem;
};

// 16-CTA clusters are a non-portable size: opt in once per kernel.
cudaError_t allow_big_clusters(const void* kernel) {
  static std::mutex mu;
  static std::vector<const void*> done;
  std::lock_guard<std::mutex> lock(mu);
  for (const void* k : done)
    if (k == kernel) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess) done.push_back(kernel);
  return e;
}

template <class G>
size_t tc_smem_bytes(int nch) {
  return 1024 + (size_t)G::kStages * 2 * nch * G::kChunk + (size_t)G::kWSmem +
         ((size_t)G::kStages * G::kRows + 2 * kEpiWarps * G::kRB + 4 * G::kRows + 8 * kComps) * 4 +
         (size_t)2 * G::kCluster * G::kRows * 8 + (size_t)G::kStages * G::kRows * 4 +
         sizeof(SmemCtl) + 64;
}

template <class G>
int max_active_clusters(int C) {
  // 0: not queried yet; -1: this cluster size cannot be co-resident
  static std::atomic<int> cache[kMaxCluster + 1];
  if (cache[C].load(std::memory_order_relaxed) == 0) {
    const int max_nch = (G::kMaxFeat + 63) / 64;
    ensure_dynamic_smem(reinterpret_cast<const void*>(tc_fused_kernel<G, 0>),
                        tc_smem_bytes<G>(max_nch));
    if (C > 8 && allow_big_clusters(reinterpret_cast<const void*>(tc_fused_kernel<G, 0>)) !=
                     cudaSuccess) {
      cudaGetLastError();
      cache[C].store(-1, std::memory_order_relaxed);
      return 0;
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(C * 64, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = tc_smem_bytes<G>(max_nch);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tc_fused_kernel<G, 0>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = C > 8 ? -1 : kSms / C;  // a 16-CTA cluster must be confirmed, not assumed
    }
    cache[C].store(n < 0 ? -1 : std::min(n, kSms / C), std::memory_order_relaxed);
  }
  const int n = cache[C].load(std::memory_order_relaxed);
  return n < 0 ? 0 : n;
}

int max_active_clusters_iso(int C) {
  // 0: not queried yet
  static std::atomic<int> cache[kIsoCluster + 1];
  if (cache[C].load(std::memory_order_relaxed) == 0) {
    ensure_dynamic_smem(reinterpret_cast<const void*>(tc_iso_kernel), IsoSmem::kDynamic);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(C * 64, 1, 1);
    cfg.blockDim = dim3(kIsoThreads, 1, 1);
    cfg.dynamicSmemBytes = IsoSmem::kDynamic;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tc_iso_kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = kSms / C;
    }
    cache[C].store(std::min(n, kSms / C), std::memory_order_relaxed);
  }
  return cache[C].load(std::memory_order_relaxed);
}

cudaError_t launch_iso(const TcPlan& pl, const TcParams& p, cudaStream_t stream) {
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(tc_iso_kernel), pl.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = pl.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(pl.C * pl.clusters, 1, 1);
  cfg.blockDim = dim3(kIsoThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tc_iso_kernel, p);
}

// single_pass = false: the plan of one component block of the K > 2048 path
// (the two-phase fused kernel, never tc_iso_kernel).
TcPlan plan_tc(int variant, int64_t N, int K, int D, bool query_device,
               bool single_pass = true) {
  TcPlan pl;
  pl.diag = variant == kDiag;
  pl.cfg = pl.diag ? (D > kMaxDDiag ? kCfgDiagWide : kCfgDiag)
                  : (D > kMaxDIso ? kCfgWide : kCfgIso);
  pl.rows = with_cfg(pl.cfg, [](auto g) { return decltype(g)::kRows; });
  // cluster size: a power of two
  pl.C = 1;
  while (pl.C * kComps < K) pl.C *= 2;
  pl.Kpad = pl.C * kComps;
  pl.Dp = (D + 15) / 16 * 16;
  pl.nfeat = pl.diag ? 2 * pl.Dp : pl.Dp;
  pl.nch = (pl.nfeat + 63) / 64;
  pl.num_tiles = (int)((N + pl.rows - 1) / pl.rows);
  pl.plen = pl.diag ? 1 + 2 * D : D + 2;
  pl.stage_bytes = (size_t)2 * pl.nch * pl.rows * 128;
  const int nch = pl.nch, C = pl.C;
  pl.big = pl.C > 8;
  pl.smem = with_cfg(pl.cfg, [nch](auto g) { return tc_smem_bytes<decltype(g)>(nch); }, pl.big);
  pl.iso = single_pass && !pl.diag && pl.cfg == kCfgIso && !pl.big;
  if (pl.iso) pl.smem = IsoSmem::kDynamic;
  int maxc = kSms / pl.C;
  if (query_device && pl.iso)
    maxc = max_active_clusters_iso(C);
  else if (query_device && pl.C <= kMaxCluster)
    maxc = with_cfg(pl.cfg, [C](auto g) { return max_active_clusters<decltype(g)>(C); }, pl.big);
  pl.clusters = std::max(1, std::min(maxc, pl.num_tiles));
  return pl;
}

// Large calls run in kChunks row chunks so the split pass of chunk c+1
// (low-priority stream) overlaps the fused kernel of chunk c (high-priority
// stream, which the fused CTAs need to get their SMs first); the split pass
// then uses the SMs the clusters leave free.  The chunks grow (1/8, 3/8, 1/2
// of the tiles): only the first, short split is exposed, and each later split
// has a longer fused kernel to hide behind on the few free SMs.  Smaller
// calls (and the whole path's workspace-free entry, which stays far below the
// threshold) run on the caller's stream alone.
constexpr int kChunks = 3;
constexpr int kChunkMinTiles = 2048;

int plan_chunks(const TcPlan& pl) { return pl.num_tiles >= kChunkMinTiles ? kChunks : 1; }
// First tile of chunk c of n (c = n gives num_tiles).
int chunk_begin(int c, int n, int num_tiles) {
  if (n == 1) return c == 0 ? 0 : num_tiles;
  static const int kEighths[kChunks + 1] = {0, 1, 4, 8};
  return (int)((int64_t)num_tiles * kEighths[c] / 8);
}

struct SideStreams {
  bool ready = false;
  cudaStream_t hi = nullptr, lo = nullptr;
  cudaEvent_t ev[kChunks + 5] = {};
};
// Per host thread and device: calls from different threads never share
// streams or events.
thread_local SideStreams t_side[16];

SideStreams* side_streams() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) return nullptr;
  SideStreams& ss = t_side[dev];
  if (!ss.ready) {
    int least = 0, greatest = 0;
    if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) return nullptr;
    if (cudaStreamCreateWithPriority(&ss.hi, cudaStreamNonBlocking, greatest) != cudaSuccess)
      return nullptr;
    if (cudaStreamCreateWithPriority(&ss.lo, cudaStreamNonBlocking, least) != cudaSuccess)
      return nullptr;
    for (auto& e : ss.ev)
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
    ss.ready = true;
  }
  return &ss;
}

template <class G>
cudaError_t launch_fused(const TcPlan& pl, const TcParams& p, cudaStream_t stream, int mode = 0) {
  void (*kern)(const TcParams) = tc_fused_kernel<G, 0>;
  if constexpr (G::kCluster <= 8) {
    if (mode == 1) kern = tc_fused_kernel<G, 1>;
    if (mode == 2) kern = tc_fused_kernel<G, 2>;
  } else if (mode != 0) {
    return cudaErrorInvalidValue;  // the 16-CTA instantiations run the single pass only
  }
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), pl.smem);
  if (e != cudaSuccess) return e;
  if constexpr (G::kCluster > 8) {
    e = allow_big_clusters(reinterpret_cast<const void*>(kern));
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = pl.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(pl.C * pl.clusters, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// Room for pairs to refine: two per row on average (a row has at most 256
// pairs with r >= 2^-8; pairs beyond the room keep the tensor-core value).
inline int64_t refine_cap(int64_t N) { return std::min<int64_t>(2 * N + 4096, INT32_MAX); }

// K > 1024 (iso / diag): the components run in blocks of 1024 (one 8-CTA
// cluster each).  Phase 1 launches the fused kernel in LSE-only mode per
// block, a small kernel combines the blocks' log-sum-exps into logZ, and
// phase 2 launches it per block with that logZ (no exchange) to form the
// statistics; the distance GEMM runs twice, the statistics once.
struct MbWs {
  int nb = 0;
  int Kb[kMaxBlocks];
  TcPlan pl[kMaxBlocks];
  int* err = nullptr;
  float* cvec = nullptr;
  __half* Whi[kMaxBlocks];
  __half* Wlo[kMaxBlocks];
  float4* consts[kMaxBlocks];  // block b at consts_all + b * kBlockComps
  float4* consts_all = nullptr;
  float* part[kMaxBlocks];
  uint8_t* xsplit = nullptr;
  float* xsq = nullptr;
  float* lse_part = nullptr;
  float* lz2 = nullptr;
  // isotropic logZ refinement: |mu_k - c| (by the call's component number),
  // per-row correction sums and the listed pairs
  float* mc = nullptr;
  unsigned long long* corr = nullptr;
  int4* refine = nullptr;
  int64_t npad = 0;
  size_t bytes = 0;
};

MbWs carve_mb(void* base, int variant, int64_t N, int K, int D, bool query_device) {
  MbWs m;
  m.nb = (K + kBlockComps - 1) / kBlockComps;
  for (int b = 0; b < m.nb; ++b) {
    m.Kb[b] = std::min(kBlockComps, K - b * kBlockComps);
    m.pl[b] = plan_tc(variant, N, m.Kb[b], D, query_device, false);
  }
  const TcPlan& p0 = m.pl[0];
  m.npad = (int64_t)p0.num_tiles * p0.rows;
  WsCarve w(base);
  m.err = w.take<int>(64);
  m.cvec = w.take<float>(p0.Dp);
  // the blocks' component constants in one array (Kpad <= kBlockComps per
  // block), so the logZ refinement indexes them by the call's component
  m.consts_all = w.take<float4>((size_t)m.nb * kBlockComps);
  for (int b = 0; b < m.nb; ++b) {
    m.Whi[b] = w.take<__half>((size_t)m.pl[b].Kpad * p0.nfeat);
    m.Wlo[b] = w.take<__half>((size_t)m.pl[b].Kpad * p0.nfeat);
    m.consts[b] = m.consts_all + (size_t)b * kBlockComps;
    m.part[b] = w.take<float>((size_t)(kSms / m.pl[b].C) * m.pl[b].Kpad * p0.plen);
  }
  m.xsplit = w.take<uint8_t>((size_t)p0.num_tiles * p0.stage_bytes);
  if (!p0.diag) m.xsq = w.take<float>((size_t)p0.num_tiles * p0.rows);
  m.lse_part = w.take<float>((size_t)m.nb * m.npad);
  m.lz2 = w.take<float>((size_t)m.npad);
  if (!p0.diag) {
    m.mc = w.take<float>((size_t)m.nb * kBlockComps);
    m.corr = w.take<unsigned long long>((size_t)N);
    m.refine = w.take<int4>((size_t)refine_cap(N));
  }
  m.bytes = w.used + 256;
  return m;
}

cudaError_t tc_estep_blocks(int variant, const EstepArgs& a) {
  const MbWs m = carve_mb(a.ws, variant, a.N, a.K, a.D, true);
  const TcPlan& p0 = m.pl[0];
  cudaStream_t st = a.stream;
  // err[3]: pairs listed for the logZ refinement (isotropic)
  const bool refine_on = !p0.diag && a.N <= INT32_MAX;  // pairs store 32-bit row numbers
  cudaError_t e = cudaMemsetAsync(m.err, 0, 4 * sizeof(int), st);
  if (e != cudaSuccess) return e;
  int launches = 0;
  // one centre and X scale for all blocks
  launch_centre(a, p0.Dp, m.cvec, m.err + 1, st);
  ++launches;
  for (int b = 0; b < m.nb; ++b) {
    const int64_t k0 = (int64_t)b * kBlockComps;
    const float* mub = a.mu + k0 * a.smk;
    if (p0.diag)
      tc_prep_diag_kernel<<<m.pl[b].Kpad, 128, 0, st>>>(mub, a.smk, a.smd, a.cov + k0 * a.D,
                                                        a.lpi + k0, m.cvec, m.err + 1, m.Kb[b],
                                                        a.D, p0.Dp, m.Whi[b], m.Wlo[b],
                                                        m.consts[b]);
    else
      tc_prep_kernel<<<m.pl[b].Kpad, prep_threads(p0.Dp), 0, st>>>(
          mub, a.smk, a.smd, a.cov + k0, a.lpi + k0, m.cvec, m.Kb[b], a.D, p0.Dp, m.Whi[b],
          m.Wlo[b], m.consts[b], nullptr, m.mc != nullptr ? m.mc + k0 : nullptr);
    ++launches;
  }
  const int vec_ok = a.x_vec_ok();
  const int sblocks =
      (int)std::min<int64_t>((m.npad + 8 * kSplitRows - 1) / (8 * kSplitRows), 16 * kSms);
  with_cfg(p0.cfg, [&](auto g) {
    return with_xtype(a.xtype, [&](auto tx) {
      using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
      tc_split_kernel<decltype(g), TX><<<sblocks, 256, 0, st>>>(
          a.x<TX>(), a.sxn, a.sxd, vec_ok, a.N, a.D, p0.Dp, p0.nch, m.npad, m.err + 1, m.cvec,
          m.xsplit, m.xsq, m.err, refine_on ? m.corr : nullptr);
      return 0;
    });
  });
  ++launches;

  TcParams p;
  p.xsplit = m.xsplit;
  p.xsq = m.xsq;
  p.N = a.N;
  p.D = a.D;
  p.Dp = p0.Dp;
  p.nfeat = p0.nfeat;
  p.nch = p0.nch;
  p.num_tiles = p0.num_tiles;
  p.xscale = m.err + 1;
  p.plen = p0.plen;
  p.err = m.err;
  if (refine_on) {  // pairs are listed by the statistics phase (mode 2)
    p.refine = m.refine;
    p.refine_count = m.err + 3;
    p.refine_cap = (int)refine_cap(a.N);
  }
  profile_mark(false, st);
  for (int phase = 1; phase <= 2; ++phase) {
    for (int b = 0; b < m.nb; ++b) {
      p.K = m.Kb[b];
      p.C = m.pl[b].C;
      p.Whi = m.Whi[b];
      p.Wlo = m.Wlo[b];
      p.consts = m.consts[b];
      p.comp_base = b * kBlockComps;
      if (refine_on) p.mc = m.mc + (size_t)b * kBlockComps;
      p.part = m.part[b];
      p.logZ = phase == 1 ? m.lse_part + (size_t)b * m.npad : m.lz2;  // out / in, log2 units
      const TcPlan& pb = m.pl[b];
      e = with_cfg(p0.cfg, [&](auto g) { return launch_fused<decltype(g)>(pb, p, st, phase); });
      if (e != cudaSuccess) return e;
      ++launches;
    }
    if (phase == 1) {
      const int cblocks = (int)std::min<int64_t>((a.N + 255) / 256, 16 * kSms);
      tc_lse_combine_kernel<<<cblocks, 256, 0, st>>>(m.lse_part, m.nb, m.npad, a.N, m.lz2,
                                                     a.logZ);
      ++launches;
    }
  }
  profile_mark(true, st);
  const int accumulate = (a.flags & 1u) ? 1 : 0;
  for (int b = 0; b < m.nb; ++b) {
    const int64_t k0 = (int64_t)b * kBlockComps;
    if (p0.diag) {
      const int64_t total = (int64_t)m.Kb[b] * (a.D + 1);
      const int rblocks = (int)std::min<int64_t>((total + 255) / 256, 1024);
      tc_reduce_diag_kernel<<<rblocks, 256, 0, st>>>(
          m.part[b], m.pl[b].clusters, m.pl[b].Kpad, m.Kb[b], a.D, m.cvec, a.mu + k0 * a.smk,
          a.smk, a.smd, m.err, a.Nk + k0, a.mu_acc + k0 * a.D, a.sig + k0 * a.D, accumulate);
    } else {
      tc_reduce_kernel<<<m.Kb[b], reduce_threads(a.D), 0, st>>>(m.part[b], m.pl[b].clusters, m.pl[b].Kpad,
                                                 m.Kb[b], a.D, m.cvec, m.err, a.Nk + k0,
                                                 a.mu_acc + k0 * a.D, a.sig + k0, accumulate);
    }
    ++launches;
  }
  if (refine_on) {
    with_xtype(a.xtype, [&](auto tx) {
      using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
      tc_refine_iso_kernel<TX><<<2 * kSms, 256, 0, st>>>(m.refine, m.err + 3, p.refine_cap,
                                                         a.x<TX>(), a.sxn, a.sxd, a.mu, a.smk,
                                                         a.smd, a.D, m.consts_all, m.corr);
      return 0;
    });
    tc_apply_refine_kernel<<<kSms, 256, 0, st>>>(m.refine, m.err + 3, p.refine_cap, m.corr,
                                                 a.logZ);
    launches += 2;
  }
  count_launches(launches);
  return cudaGetLastError();
}

}  // namespace

// ---------------------------------------------------------------------------
// Centre, one block per feature d (Dp blocks of 256 threads):
// c_d = mean_k mu_kd (0 for padding features) and amax = max of |mu_kd - c_d|
// and of |x_nd - c_d| over a sample of rows (the X scale of the split passes).
// Centring by one global vector leaves every x - mu_k unchanged and keeps
// expanded forms (x^2 - 2 x mu + mu^2, x L - mu L, x x^T) away from
// cancellation when the data sit far from the origin.
// ---------------------------------------------------------------------------
template <class TX>
__global__ void __launch_bounds__(256) centre_kernel(const float* __restrict__ mu,
                                                             int64_t smk, int64_t smd, int K,
                                                             int D, const TX* __restrict__ X,
                                                             int64_t sxn, int64_t sxd, int64_t N,
                                                             float* __restrict__ cvec,
                                                             int* __restrict__ amax) {
  const int d = blockIdx.x;
  __shared__ double s_sum[8];
  __shared__ float s_max[8];
  __shared__ float s_c;
  double sum = 0.0;
  if (d < D) {
#pragma unroll 4
    for (int k = threadIdx.x; k < K; k += 256) sum += (double)mu[(int64_t)k * smk + (int64_t)d * smd];
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) s_sum[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += s_sum[w];
    s_c = d < D ? (float)(t / K) : 0.f;
    cvec[d] = s_c;
  }
  __syncthreads();
  const float c = s_c;
  float mx = 0.f;
  if (d < D) {
#pragma unroll 4
    for (int k = threadIdx.x; k < K; k += 256)
      mx = fmaxf(mx, fabsf(mu[(int64_t)k * smk + (int64_t)d * smd] - c));
    // and over an evenly spaced sample of up to kScaleSample rows of X, so the
    // scale also covers the data when the means sit close together (K = 1,
    // means near the global mean)
    const int64_t ns = N < kScaleSample ? N : kScaleSample;
    for (int64_t i = threadIdx.x; i < ns; i += 256) {
      const int64_t n = i * N / ns;
      mx = fmaxf(mx, fabsf(ldx(X + n * sxn + (int64_t)d * sxd) - c));
    }
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int w = 0; w < 8; ++w) m = fmaxf(m, s_max[w]);
    atomicMax(amax, __float_as_int(m));
  }
}

void launch_centre(const EstepArgs& a, int Dp, float* cvec, int* amax, cudaStream_t stream) {
  with_xtype(a.xtype, [&](auto tx) {
    using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
    centre_kernel<TX><<<Dp, 256, 0, stream>>>(a.mu, a.smk, a.smd, a.K, a.D, a.x<TX>(), a.sxn,
                                              a.sxd, a.N, cvec, amax);
    return 0;
  });
}


bool tc_supported(int variant, const EstepArgs& a, std::string* why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (variant == kIso) {
    if (a.D > kMaxDIsoWide) return no("D > 256");
  } else if (variant == kDiag) {
    if (a.D > kMaxDDiagWide) return no("D > 128");
  } else {
    return full_tc_supported(a) ? true : no("full covariance: D > 64 or scratch too large");
  }
  if (a.K > kMaxBlocks * kBlockComps) return no("K > 16384");
  return true;
}

size_t tc_workspace_bytes(int variant, int64_t N, int K, int D) {
  if (variant == kFull) return full_tc_workspace_bytes(N, K, D);
  EstepArgs probe{};
  probe.K = K;
  probe.D = D;
  if (!tc_supported(variant, probe, nullptr)) return 0;
  if (K > 2 * kBlockComps) return carve_mb(nullptr, variant, N, K, D, false).bytes;
  // 1024 < K <= 2048: one pass on 16-CTA clusters where the device can hold
  // them, else the blocked path; the workspace covers either
  const size_t blocked = K > kBlockComps ? carve_mb(nullptr, variant, N, K, D, false).bytes : 0;
  TcPlan pl = plan_tc(variant, N, K, D, false);
  WsCarve w(nullptr);
  w.take<int>(64);
  w.take<float>(pl.Dp);                                                // centre c
  w.take<__half>((size_t)pl.Kpad * pl.nfeat);
  w.take<__half>((size_t)pl.Kpad * pl.nfeat);
  w.take<float4>(pl.Kpad);
  // partial rows for the largest cluster count a 148-SM device can run,
  // per row chunk when the call is split into chunks
  w.take<float>((size_t)plan_chunks(pl) * (kSms / pl.C) * pl.Kpad * pl.plen);
  w.take<uint8_t>((size_t)pl.num_tiles * pl.stage_bytes);             // split features
  if (!pl.diag) w.take<float>((size_t)pl.num_tiles * pl.rows);         // |x|^2
  if (!pl.diag) {                                                      // logZ refinement
    w.take<float>(pl.Kpad);
    w.take<unsigned long long>((size_t)N);
    w.take<int4>((size_t)refine_cap(N));
  }
  return std::max(w.used + 256, blocked);
}

cudaError_t tc_estep(int variant, const EstepArgs& a) {
  if (variant == kFull) return full_tc_estep(a);
  if (a.K > 2 * kBlockComps) return tc_estep_blocks(variant, a);
  TcPlan pl = plan_tc(variant, a.N, a.K, a.D, true);
  if (pl.big) {  // 1024 < K <= 2048: one pass if 16-CTA clusters fit on this device
    const int C = pl.C;
    const int n = with_cfg(pl.cfg, [C](auto g) { return max_active_clusters<decltype(g)>(C); },
                           true);
    if (n <= 0) return tc_estep_blocks(variant, a);
  }
  WsCarve w(a.ws);
  int* err = w.take<int>(64);
  float* cvec = w.take<float>(pl.Dp);
  __half* Whi = w.take<__half>((size_t)pl.Kpad * pl.nfeat);
  __half* Wlo = w.take<__half>((size_t)pl.Kpad * pl.nfeat);
  float4* consts = w.take<float4>(pl.Kpad);
  int nchunks = plan_chunks(pl);
  float* part = w.take<float>((size_t)nchunks * (kSms / pl.C) * pl.Kpad * pl.plen);
  uint8_t* xsplit = w.take<uint8_t>((size_t)pl.num_tiles * pl.stage_bytes);
  float* xsq = pl.diag ? nullptr : w.take<float>((size_t)pl.num_tiles * pl.rows);
  float* mc = nullptr;
  unsigned long long* corr = nullptr;
  int4* refine = nullptr;
  const bool refine_on = !pl.diag && a.N <= INT32_MAX;  // pairs store 32-bit row numbers
  if (!pl.diag) {
    mc = w.take<float>(pl.Kpad);
    corr = w.take<unsigned long long>((size_t)a.N);
    refine = w.take<int4>((size_t)refine_cap(a.N));
  }

  SideStreams* ss = nchunks > 1 ? side_streams() : nullptr;
  if (ss == nullptr) nchunks = 1;
  // hi: prep, fused kernels, reduce; lo: split passes (same stream when not chunked)
  cudaStream_t hi = a.stream, lo = a.stream;
  cudaError_t e;
  if (nchunks > 1) {
    hi = ss->hi;
    lo = ss->lo;
    if ((e = cudaEventRecord(ss->ev[0], a.stream)) != cudaSuccess) return e;
    if ((e = cudaStreamWaitEvent(hi, ss->ev[0], 0)) != cudaSuccess) return e;
    if ((e = cudaStreamWaitEvent(lo, ss->ev[0], 0)) != cudaSuccess) return e;
  }

  // err[0]: device error word, err[1]: max|mu - c| (float bits, for the X
  // scale), written by the centre kernel
  // err[2]: the components' variances differ (isotropic prep)
  // err[3]: pairs listed for the logZ refinement (isotropic kernels)
  e = cudaMemsetAsync(err, 0, 4 * sizeof(int), hi);
  if (e != cudaSuccess) return e;

  int launches = 0;
  launch_centre(a, pl.Dp, cvec, err + 1, hi);
  if (nchunks > 1) {  // the split passes need c and max|mu - c| only: they overlap the prep
    if ((e = cudaEventRecord(ss->ev[1], hi)) != cudaSuccess) return e;
    if ((e = cudaStreamWaitEvent(lo, ss->ev[1], 0)) != cudaSuccess) return e;
  }
  if (pl.diag)
    tc_prep_diag_kernel<<<pl.Kpad, 128, 0, hi>>>(a.mu, a.smk, a.smd, a.cov, a.lpi, cvec, err + 1,
                                                 a.K, a.D, pl.Dp, Whi, Wlo, consts);
  else
    tc_prep_kernel<<<pl.Kpad, prep_threads(pl.Dp), 0, hi>>>(a.mu, a.smk, a.smd, a.cov, a.lpi, cvec, a.K, a.D,
                                            pl.Dp, Whi, Wlo, consts, err + 2, mc);
  launches += 2;
  const int vec_ok = a.x_vec_ok();

  // split passes (stream lo), one per chunk of tiles [t0, t1)
  for (int c = 0; c < nchunks; ++c) {
    const int t0 = chunk_begin(c, nchunks, pl.num_tiles);
    const int t1 = chunk_begin(c + 1, nchunks, pl.num_tiles);
    if (t0 >= t1) break;
    const int64_t row0 = (int64_t)t0 * pl.rows;
    const int64_t rows = std::min<int64_t>(a.N, (int64_t)t1 * pl.rows) - row0;
    const int64_t rows_pad = (int64_t)(t1 - t0) * pl.rows;
    const int sblocks =
        (int)std::min<int64_t>((rows_pad + 8 * kSplitRows - 1) / (8 * kSplitRows), 16 * kSms);
    uint8_t* xs_c = xsplit + (size_t)t0 * pl.stage_bytes;
    float* xsq_c = pl.diag ? nullptr : xsq + (size_t)t0 * pl.rows;
    with_cfg(pl.cfg, [&](auto g) {
      return with_xtype(a.xtype, [&](auto tx) {
        using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
        const TX* Xc = a.x<TX>() + row0 * a.sxn;
        tc_split_kernel<decltype(g), TX><<<sblocks, 256, 0, lo>>>(
            Xc, a.sxn, a.sxd, vec_ok, rows, a.D, pl.Dp, pl.nch, rows_pad, err + 1, cvec, xs_c,
            xsq_c, err, refine_on ? corr + row0 : nullptr);
        return 0;
      });
    });
    ++launches;
    if (nchunks > 1 && (e = cudaEventRecord(ss->ev[2 + c], lo)) != cudaSuccess) return e;
  }

  // fused kernels (stream hi), each after its chunk's split; partials of
  // chunk c follow those of chunks < c, so one reduction sums them in order
  TcParams p;
  p.K = a.K;
  p.D = a.D;
  p.Dp = pl.Dp;
  p.nfeat = pl.nfeat;
  p.nch = pl.nch;
  p.C = pl.C;
  p.Whi = Whi;
  p.Wlo = Wlo;
  p.consts = consts;
  p.xscale = err + 1;
  p.nonuniform = pl.diag ? nullptr : err + 2;
  p.plen = pl.plen;
  p.err = err;
  if (refine_on) {
    p.mc = mc;
    p.refine = refine;
    p.refine_count = err + 3;
    p.refine_cap = (int)refine_cap(a.N);
  }
  int part_clusters = 0, presummed = 0;
  for (int c = 0; c < nchunks; ++c) {
    const int t0 = chunk_begin(c, nchunks, pl.num_tiles);
    const int t1 = chunk_begin(c + 1, nchunks, pl.num_tiles);
    if (t0 >= t1) break;
    if (nchunks > 1 && (e = cudaStreamWaitEvent(hi, ss->ev[2 + c], 0)) != cudaSuccess) return e;
    if (c == 0) profile_mark(false, hi);  // the fused kernels of all chunks are bracketed
    const int64_t row0 = (int64_t)t0 * pl.rows;
    TcPlan pc = pl;
    pc.num_tiles = t1 - t0;
    pc.clusters = std::max(1, std::min(pl.clusters, pc.num_tiles));
    p.xsplit = xsplit + (size_t)t0 * pl.stage_bytes;
    p.xsq = pl.diag ? nullptr : xsq + (size_t)t0 * pl.rows;
    p.N = std::min<int64_t>(a.N, (int64_t)t1 * pl.rows) - row0;
    p.num_tiles = pc.num_tiles;
    p.logZ = a.logZ + row0;
    p.row_base = (int)row0;
    p.part = part + (size_t)part_clusters * pl.Kpad * pl.plen;
    if (pl.iso)
      e = launch_iso(pc, p, hi);
    else
      e = with_cfg(pl.cfg, [&](auto g) { return launch_fused<decltype(g)>(pc, p, hi); }, pl.big);
    if (e != cudaSuccess) return e;
    part_clusters += pc.clusters;
    ++launches;
    if (nchunks > 1 && c == nchunks - 2) {
      // pre-sum the partials so far on the side stream, behind the last chunk
      const int64_t slot = (int64_t)pl.Kpad * pl.plen;
      if ((e = cudaEventRecord(ss->ev[3 + kChunks], hi)) != cudaSuccess) return e;
      if ((e = cudaStreamWaitEvent(lo, ss->ev[3 + kChunks], 0)) != cudaSuccess) return e;
      tc_part_presum_kernel<<<(int)std::min<int64_t>((slot + 255) / 256, 4 * kSms), 256, 0, lo>>>(
          part, part_clusters, slot);
      ++launches;
      if ((e = cudaEventRecord(ss->ev[4 + kChunks], lo)) != cudaSuccess) return e;
      presummed = part_clusters - 1;
    }
  }
  profile_mark(true, hi);
  if (presummed > 0) {
    if ((e = cudaStreamWaitEvent(hi, ss->ev[4 + kChunks], 0)) != cudaSuccess) return e;
    part += (size_t)presummed * pl.Kpad * pl.plen;
    part_clusters -= presummed;
  }
  const int accumulate = (a.flags & 1u) ? 1 : 0;
  if (pl.diag) {
    const int64_t total = (int64_t)a.K * (a.D + 1);
    const int rblocks = (int)std::min<int64_t>((total + 255) / 256, 1024);
    tc_reduce_diag_kernel<<<rblocks, 256, 0, hi>>>(part, part_clusters, pl.Kpad, a.K, a.D, cvec,
                                                   a.mu, a.smk, a.smd, err, a.Nk, a.mu_acc,
                                                   a.sig, accumulate);
  } else {
    tc_reduce_kernel<<<a.K, reduce_threads(a.D), 0, hi>>>(part, part_clusters, pl.Kpad, a.K, a.D, cvec, err, a.Nk,
                                          a.mu_acc, a.sig, accumulate);
  }
  ++launches;
  if (refine_on) {
    with_xtype(a.xtype, [&](auto tx) {
      using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
      tc_refine_iso_kernel<TX><<<2 * kSms, 256, 0, hi>>>(refine, err + 3, p.refine_cap, a.x<TX>(),
                                                         a.sxn, a.sxd, a.mu, a.smk, a.smd, a.D,
                                                         consts, corr);
      return 0;
    });
    tc_apply_refine_kernel<<<kSms, 256, 0, hi>>>(refine, err + 3, p.refine_cap, corr, a.logZ);
    launches += 2;
  }
  count_launches(launches);
  if (nchunks > 1) {
    if ((e = cudaEventRecord(ss->ev[2 + kChunks], hi)) != cudaSuccess) return e;
    if ((e = cudaStreamWaitEvent(a.stream, ss->ev[2 + kChunks], 0)) != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

}  // namespace fgmm
