// General E-step kernels on the CUDA cores (fp32 FMA, exact differences).
//
// These handle every shape and stride the C ABI accepts (D <= 256 for the
// isotropic / diagonal families, D <= 128 for full covariance) and are the
// path the tensor-core kernels fall back to outside their envelope.  They
// follow the reference's two-pass structure -- a per-row online log-sum-exp
// (flash_gmm.py:50-103) and a responsibilities/statistics pass
// (flash_gmm.py:110-166) -- but compute ||x - mu||^2 by differences instead of
// the x^2 - 2 x.mu + mu^2 expansion (flash_gmm.py:84-88), and replace the
// global atomics with per-block partial sums reduced in a fixed order.
#include <math.h>

#include <algorithm>
#include <type_traits>

#include "fgmm_internal.cuh"

namespace fgmm {
namespace {

constexpr int kThreads = 256;
constexpr int BR = 64;   // rows per tile
constexpr int BC = 64;   // components per tile
constexpr int DC = 32;   // feature chunk of the distance loop
constexpr int PAD = 4;

__device__ __forceinline__ float warp16_max(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp16_sum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// Per-component constants.
//   iso : cst_k = log_pi_k - D/2 (log 2pi + lss_k), inv_k = exp(-lss_k)
//         (flash_gmm.py:90-92)
//   diag: cst_k = log_pi_k - 1/2 (D log 2pi + sum_d lss_kd), inv_kd = exp(-lss_kd)
//         (flash_gmm_diag_h100.py:332-339)
//   full: cst_k = log_pi_k + sum_d log(|L_kdd| + 1e-30) - D/2 log 2pi
//         (flash_gmm_full_h100.py:294-296)
// ---------------------------------------------------------------------------
__global__ void prep_kernel(int variant, const float* __restrict__ cov,
                            const float* __restrict__ lpi, int K, int D,
                            float* __restrict__ cst, float* __restrict__ inv) {
  int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= K) return;
  double lp = (double)lpi[k];
  if (variant == kIso) {
    double l = (double)cov[k];
    cst[k] = (float)(lp - 0.5 * D * (kLog2Pi + l));
    inv[k] = (float)exp(-l);
  } else if (variant == kDiag) {
    double s = 0.0;
    for (int d = 0; d < D; ++d) {
      double l = (double)cov[(size_t)k * D + d];
      s += l;
      inv[(size_t)k * D + d] = (float)exp(-l);
    }
    cst[k] = (float)(lp - 0.5 * (D * kLog2Pi + s));
  } else {
    double s = 0.0;
    for (int d = 0; d < D; ++d)
      s += log(fabs((double)cov[((size_t)k * D + d) * D + d]) + 1e-30);
    cst[k] = (float)(lp + s - 0.5 * D * kLog2Pi);
  }
}

// Distance tile: acc[i][j] = sum_d (x_{row i} - mu_{comp j})^2 [* inv_{comp j, d}]
// for the 64x64 tile (rows row0.., comps c0..); thread (ty, tx) owns rows
// ty*4+i and components tx*4+j.
template <bool DIAG, class TX>
__device__ __forceinline__ void distance_tile(
    const TX* __restrict__ X, int64_t sxn, int64_t sxd, const float* __restrict__ mu,
    int64_t smk, int64_t smd, const float* __restrict__ inv, int64_t N, int K, int D,
    int64_t row0, int c0, float (*xs)[BR + PAD], float (*ms)[BC + PAD],
    float (*is)[BC + PAD], float acc[4][4]) {
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int d0 = 0; d0 < D; d0 += DC) {
    for (int e = tid; e < BR * DC; e += kThreads) {
      int r = e / DC, d = e % DC;
      int64_t row = row0 + r;
      int dd = d0 + d;
      xs[d][r] = (row < N && dd < D) ? ldx(X + (row * sxn + (int64_t)dd * sxd)) : 0.f;
    }
    for (int e = tid; e < BC * DC; e += kThreads) {
      int c = e / DC, d = e % DC;
      int cc = c0 + c, dd = d0 + d;
      bool ok = cc < K && dd < D;
      ms[d][c] = ok ? mu[(int64_t)cc * smk + (int64_t)dd * smd] : 0.f;
      if (DIAG) is[d][c] = ok ? inv[(size_t)cc * D + dd] : 0.f;
    }
    __syncthreads();
    const int dlim = min(DC, D - d0);
    for (int d = 0; d < dlim; ++d) {
      float4 xv = *reinterpret_cast<const float4*>(&xs[d][ty * 4]);
      float4 mv = *reinterpret_cast<const float4*>(&ms[d][tx * 4]);
      float x4[4] = {xv.x, xv.y, xv.z, xv.w};
      float m4[4] = {mv.x, mv.y, mv.z, mv.w};
      if (DIAG) {
        float4 iv = *reinterpret_cast<const float4*>(&is[d][tx * 4]);
        float i4[4] = {iv.x, iv.y, iv.z, iv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float df = x4[i] - m4[j];
            acc[i][j] = fmaf(df * df, i4[j], acc[i][j]);
          }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float df = x4[i] - m4[j];
            acc[i][j] = fmaf(df, df, acc[i][j]);
          }
      }
    }
    __syncthreads();
  }
}

// ll = cst_k - 1/2 inv_k sq (iso) or cst_k - 1/2 quad (diag); -inf outside K.
template <bool DIAG>
__device__ __forceinline__ float loglik(float q, int c, int K, const float* __restrict__ cst,
                                        const float* __restrict__ inv) {
  if (c >= K) return -INFINITY;
  return DIAG ? fmaf(-0.5f, q, cst[c]) : fmaf(-0.5f * inv[c], q, cst[c]);
}

// ---------------------------------------------------------------------------
// Pass 1 (iso / diag): logZ per row by an online log-sum-exp over component
// tiles (flash_gmm.py:72-103).
// ---------------------------------------------------------------------------
template <bool DIAG, class TX>
__global__ void __launch_bounds__(kThreads) lse_kernel(
    const TX* __restrict__ X, int64_t sxn, int64_t sxd, const float* __restrict__ mu,
    int64_t smk, int64_t smd, const float* __restrict__ inv, const float* __restrict__ cst,
    int64_t N, int K, int D, float* __restrict__ logZ) {
  __shared__ __align__(16) float xs[DC][BR + PAD];
  __shared__ __align__(16) float ms[DC][BC + PAD];
  __shared__ __align__(16) float is[DIAG ? DC : 1][BC + PAD];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t row0 = (int64_t)blockIdx.x * BR;
  float run_m[4], run_s[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) { run_m[i] = -INFINITY; run_s[i] = 0.f; }
  for (int c0 = 0; c0 < K; c0 += BC) {
    float acc[4][4];
    distance_tile<DIAG>(X, sxn, sxd, mu, smk, smd, inv, N, K, D, row0, c0, xs, ms, is, acc);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float ll[4];
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ll[j] = loglik<DIAG>(acc[i][j], c0 + tx * 4 + j, K, cst, inv);
        m = fmaxf(m, ll[j]);
      }
      m = warp16_max(m);
      const float nm = fmaxf(run_m[i], m);
      float s = 0.f;
      if (nm > -INFINITY) {
#pragma unroll
        for (int j = 0; j < 4; ++j) s += expf(ll[j] - nm);
      }
      s = warp16_sum(s);
      run_s[i] = (nm > -INFINITY) ? fmaf(run_s[i], expf(run_m[i] - nm), s) : 0.f;
      run_m[i] = nm;
    }
  }
  if (tx == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int64_t row = row0 + ty * 4 + i;
      if (row < N) logZ[row] = run_m[i] + logf(run_s[i]);
    }
  }
}

// ---------------------------------------------------------------------------
// Pass 2 (iso / diag): per (component tile, row slab) block, responsibilities
// r = exp(ll - logZ) (flash_gmm.py:151) and the block's partial statistics
//   part[slab][k] = { Nk, sig_or_unused, mu_acc[0..D), x2acc[0..D) (diag) }
// accumulated over the slab's rows.  The slab partition is exact (no row is
// visited twice; cf. the overlap at flash_gmm_diag_h100.py:220-236).
// Dynamic shared memory: acc_mu[BC][D], (diag) acc_x2[BC][D].
// ---------------------------------------------------------------------------
template <bool DIAG, class TX>
__global__ void __launch_bounds__(kThreads) stats_kernel(
    const TX* __restrict__ X, int64_t sxn, int64_t sxd, const float* __restrict__ mu,
    int64_t smk, int64_t smd, const float* __restrict__ inv, const float* __restrict__ cst,
    int64_t N, int K, int D, const float* __restrict__ logZ, int64_t rows_per_slab,
    int part_len, float* __restrict__ part) {
  extern __shared__ __align__(16) float dyn[];
  float (*xs)[BR + PAD] = reinterpret_cast<float (*)[BR + PAD]>(dyn);
  float (*ms)[BC + PAD] = reinterpret_cast<float (*)[BC + PAD]>(dyn + DC * (BR + PAD));
  float (*is)[BC + PAD] = reinterpret_cast<float (*)[BC + PAD]>(dyn + 2 * DC * (BR + PAD));
  float (*rs)[BC + PAD] = reinterpret_cast<float (*)[BC + PAD]>(dyn + 3 * DC * (BR + PAD));
  float (*ws)[BC + PAD] = rs + BR;  // r * sq (iso)
  float (*xc)[BC + PAD] = ws + BR;  // feature chunk of 64 for R^T X
  float* acc_mu = &xc[BR][0];                 // [BC][D]
  float* acc_x2 = acc_mu + (size_t)BC * D;    // [BC][D] (diag)

  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int c0 = blockIdx.x * BC;
  const int64_t r_begin = (int64_t)blockIdx.y * rows_per_slab;
  const int64_t r_end = min(N, r_begin + rows_per_slab);

  for (int e = tid; e < BC * D * (DIAG ? 2 : 1); e += kThreads) acc_mu[e] = 0.f;
  float nk_run = 0.f, sig_run = 0.f;  // owned by threads tid < BC
  __syncthreads();

  for (int64_t row0 = r_begin; row0 < r_end; row0 += BR) {
    float acc[4][4];
    distance_tile<DIAG>(X, sxn, sxd, mu, smk, smd, inv, r_end, K, D, row0, c0, xs, ms, is, acc);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rl = ty * 4 + i;
      const int64_t row = row0 + rl;
      const float lz = row < r_end ? logZ[row] : 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int cl = tx * 4 + j;
        float ll = loglik<DIAG>(acc[i][j], c0 + cl, K, cst, inv);
        float r = (row < r_end && ll > -INFINITY) ? expf(ll - lz) : 0.f;
        rs[rl][cl] = r;
        ws[rl][cl] = r * acc[i][j];
      }
    }
    __syncthreads();
    if (tid < BC) {
      float a = 0.f, b = 0.f;
      for (int r = 0; r < BR; ++r) { a += rs[r][tid]; b += ws[r][tid]; }
      nk_run += a;
      sig_run += b;
    }
    // acc_mu[c][d] += sum_rows r[row][c] x[row][d] over feature chunks of 64;
    // thread (ty, tx) owns components ty*4+i and features tx*4+j of the chunk.
    for (int f0 = 0; f0 < D; f0 += 64) {
      for (int e = tid; e < BR * 64; e += kThreads) {
        int r = e / 64, d = e % 64;
        int64_t row = row0 + r;
        int dd = f0 + d;
        xc[r][d] = (row < r_end && dd < D) ? ldx(X + (row * sxn + (int64_t)dd * sxd)) : 0.f;
      }
      __syncthreads();
      float am[4][4], a2[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) { am[i][j] = 0.f; a2[i][j] = 0.f; }
      for (int r = 0; r < BR; ++r) {
        float4 rv = *reinterpret_cast<const float4*>(&rs[r][ty * 4]);
        float4 xv = *reinterpret_cast<const float4*>(&xc[r][tx * 4]);
        float r4[4] = {rv.x, rv.y, rv.z, rv.w};
        float x4[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            am[i][j] = fmaf(r4[i], x4[j], am[i][j]);
            if (DIAG) a2[i][j] = fmaf(r4[i] * x4[j], x4[j], a2[i][j]);
          }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int dd = f0 + tx * 4 + j;
          if (dd < D) {
            size_t o = (size_t)(ty * 4 + i) * D + dd;
            acc_mu[o] += am[i][j];
            if (DIAG) acc_x2[o] += a2[i][j];
          }
        }
      __syncthreads();
    }
  }
  // Write the block's partials: part[(slab * K + k) * part_len + ...].
  float* out = part + (size_t)blockIdx.y * K * part_len;
  if (tid < BC && c0 + tid < K) {
    out[(size_t)(c0 + tid) * part_len + 0] = nk_run;
    out[(size_t)(c0 + tid) * part_len + 1] = sig_run;
  }
  for (int e = tid; e < BC * D; e += kThreads) {
    int c = e / D, d = e % D;
    if (c0 + c < K) {
      out[(size_t)(c0 + c) * part_len + 2 + d] = acc_mu[e];
      if (DIAG) out[(size_t)(c0 + c) * part_len + 2 + D + d] = acc_x2[e];
    }
  }
}

// ---------------------------------------------------------------------------
// Full covariance.  maha_nk = ||L_k^T (x_n - mu_k)||^2 with the dense L_k
// (flash_gmm_full_h100.py:109-129 uses the dense transposed factor too).
// Block of 256 threads = 64 rows x 4 column groups; thread (rw, q) forms
// v_j = sum_i y_i L_k[i][j] for j = q, q+4, ... and its share of sum v_j^2.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float full_maha_part(const float* __restrict__ yrow,
                                                const float* __restrict__ Ls, int D, int q) {
  float s = 0.f;
  for (int j = q; j < D; j += 4) {
    float v = 0.f;
    for (int i = 0; i < D; ++i) v = fmaf(yrow[i], Ls[i * D + j], v);
    s = fmaf(v, v, s);
  }
  return s;
}

template <class TX>
__global__ void __launch_bounds__(kThreads) full_lse_kernel(
    const TX* __restrict__ X, int64_t sxn, int64_t sxd, const float* __restrict__ mu,
    int64_t smk, int64_t smd, const float* __restrict__ L, const float* __restrict__ cst,
    int64_t N, int K, int D, float* __restrict__ logZ) {
  extern __shared__ __align__(16) float dyn[];
  float* Ls = dyn;                       // [D][D]
  float* xs = Ls + (size_t)D * D;        // [BR][D+1]
  float* ys = xs + (size_t)BR * (D + 1); // [BR][D+1]
  const int tid = threadIdx.x, rw = tid >> 2, q = tid & 3;
  const int64_t row0 = (int64_t)blockIdx.x * BR;
  const int ld = D + 1;
  for (int e = tid; e < BR * D; e += kThreads) {
    int r = e / D, d = e % D;
    int64_t row = row0 + r;
    xs[r * ld + d] = row < N ? ldx(X + (row * sxn + (int64_t)d * sxd)) : 0.f;
  }
  float run_m = -INFINITY, run_s = 0.f;
  for (int k = 0; k < K; ++k) {
    __syncthreads();
    for (int e = tid; e < D * D; e += kThreads) Ls[e] = L[(size_t)k * D * D + e];
    for (int e = tid; e < BR * D; e += kThreads) {
      int r = e / D, d = e % D;
      ys[r * ld + d] = xs[r * ld + d] - mu[(int64_t)k * smk + (int64_t)d * smd];
    }
    __syncthreads();
    float s = full_maha_part(ys + rw * ld, Ls, D, q);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    const float ll = fmaf(-0.5f, s, cst[k]);
    const float nm = fmaxf(run_m, ll);
    run_s = (nm > -INFINITY) ? fmaf(run_s, expf(run_m - nm), expf(ll - nm)) : 0.f;
    run_m = nm;
  }
  const int64_t row = row0 + rw;
  if (q == 0 && row < N) logZ[row] = run_m + logf(run_s);
}

// Pass 2, full covariance: block = (component k, row slab).  Thread t owns a
// DT x DT block of sig_outer[k] (DT = D_MAX/16) and, for t < D, mu_acc[k][t].
// part[(slab*K + k)*part_len + ...] = { Nk, mu_acc[0..D), outer[0..D*D) }.
template <int DT, class TX>
__global__ void __launch_bounds__(kThreads) full_stats_kernel(
    const TX* __restrict__ X, int64_t sxn, int64_t sxd, const float* __restrict__ mu,
    int64_t smk, int64_t smd, const float* __restrict__ L, const float* __restrict__ cst,
    int64_t N, int K, int D, const float* __restrict__ logZ, int64_t rows_per_slab,
    int part_len, float* __restrict__ part) {
  extern __shared__ __align__(16) float dyn[];
  float* Ls = dyn;                        // [D][D]
  float* xs = Ls + (size_t)D * D;         // [BR][D+1]
  float* ys = xs + (size_t)BR * (D + 1);  // [BR][D+1]
  __shared__ float rsm[BR];
  const int tid = threadIdx.x, rw = tid >> 2, q = tid & 3;
  const int k = blockIdx.x;
  const int ld = D + 1;
  const int64_t r_begin = (int64_t)blockIdx.y * rows_per_slab;
  const int64_t r_end = min(N, r_begin + rows_per_slab);
  for (int e = tid; e < D * D; e += kThreads) Ls[e] = L[(size_t)k * D * D + e];
  const float ck = cst[k];
  const int bi = (tid >> 4) * DT, bj = (tid & 15) * DT;  // owned outer block
  float acc[DT][DT];
#pragma unroll
  for (int i = 0; i < DT; ++i)
#pragma unroll
    for (int j = 0; j < DT; ++j) acc[i][j] = 0.f;
  float mu_run = 0.f, nk_run = 0.f;

  for (int64_t row0 = r_begin; row0 < r_end; row0 += BR) {
    __syncthreads();
    for (int e = tid; e < BR * D; e += kThreads) {
      int r = e / D, d = e % D;
      int64_t row = row0 + r;
      float x = row < r_end ? ldx(X + (row * sxn + (int64_t)d * sxd)) : 0.f;
      xs[r * ld + d] = x;
      ys[r * ld + d] = x - mu[(int64_t)k * smk + (int64_t)d * smd];
    }
    __syncthreads();
    float s = full_maha_part(ys + rw * ld, Ls, D, q);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    const int64_t row = row0 + rw;
    if (q == 0) rsm[rw] = row < r_end ? expf(fmaf(-0.5f, s, ck) - logZ[row]) : 0.f;
    __syncthreads();
    for (int r = 0; r < BR; ++r) {
      const float rr = rsm[r];
      const float* xr = xs + r * ld;
      float xi[DT], xj[DT];
#pragma unroll
      for (int i = 0; i < DT; ++i) {
        xi[i] = (bi + i < D) ? rr * xr[bi + i] : 0.f;
        xj[i] = (bj + i < D) ? xr[bj + i] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < DT; ++i)
#pragma unroll
        for (int j = 0; j < DT; ++j) acc[i][j] = fmaf(xi[i], xj[j], acc[i][j]);
      if (tid < D) mu_run = fmaf(rr, xr[tid], mu_run);
      if (tid == 0) nk_run += rr;
    }
  }
  float* out = part + ((size_t)blockIdx.y * K + k) * part_len;
  if (tid == 0) out[0] = nk_run;
  if (tid < D) out[1 + tid] = mu_run;
#pragma unroll
  for (int i = 0; i < DT; ++i)
#pragma unroll
    for (int j = 0; j < DT; ++j)
      if (bi + i < D && bj + j < D) out[1 + D + (size_t)(bi + i) * D + bj + j] = acc[i][j];
}

// ---------------------------------------------------------------------------
// Deterministic reduction of per-slab partials into the outputs, summing the
// slabs in index order.  diag's sig is rebuilt from the raw moments as
// sum r x^2 - 2 mu sum r x + mu^2 sum r (flash_gmm_diag_h100.py:258-260).
// ---------------------------------------------------------------------------
__global__ void reduce_kernel(int variant, const float* __restrict__ part, int slabs, int K,
                              int D, int part_len, const float* __restrict__ mu, int64_t smk,
                              int64_t smd, float* __restrict__ Nk, float* __restrict__ mu_acc,
                              float* __restrict__ sig, int accumulate) {
  const int64_t total = (int64_t)K * part_len;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(e / part_len), j = (int)(e % part_len);
    if (variant == kDiag && j >= 2 + D) continue;  // consumed with its mu_acc twin
    double s = 0.0, s2 = 0.0, snk = 0.0;
    for (int sl = 0; sl < slabs; ++sl) {
      const float* p = part + ((size_t)sl * K + k) * part_len;
      s += p[j];
      if (variant == kDiag && j >= 2) { s2 += p[j + D]; snk += p[0]; }
    }
    float* dst;
    float v = (float)s;
    if (variant == kIso) {
      dst = j == 0 ? &Nk[k] : j == 1 ? &sig[k] : &mu_acc[(size_t)k * D + (j - 2)];
    } else if (variant == kDiag) {
      if (j == 1) continue;
      if (j == 0) {
        dst = &Nk[k];
      } else {
        const int d = j - 2;
        const double m = (double)mu[(int64_t)k * smk + (int64_t)d * smd];
        const float sg = (float)(s2 - 2.0 * m * s + m * m * snk);
        float* sdst = &sig[(size_t)k * D + d];
        *sdst = accumulate ? *sdst + sg : sg;
        dst = &mu_acc[(size_t)k * D + d];
      }
    } else {
      dst = j == 0 ? &Nk[k] : j <= D ? &mu_acc[(size_t)k * D + (j - 1)]
                                     : &sig[(size_t)k * D * D + (j - 1 - D)];
    }
    *dst = accumulate ? *dst + v : v;
  }
}

struct GeneralPlan {
  int slabs;
  int64_t rows_per_slab;
  int part_len;
};

GeneralPlan plan_general(int variant, int64_t N, int K, int D) {
  GeneralPlan p;
  const int target = 4 * 148;  // fixed (not queried) so the workspace size is device-independent
  const int64_t row_tiles = (N + BR - 1) / BR;
  const int col_blocks = variant == kFull ? K : (K + BC - 1) / BC;
  int64_t s = (target + col_blocks - 1) / col_blocks;
  if (s > row_tiles) s = row_tiles;
  if (s < 1) s = 1;
  const int64_t tiles_per_slab = row_tiles > 0 ? (row_tiles + s - 1) / s : 1;
  p.rows_per_slab = tiles_per_slab * BR;
  p.slabs = (int)((N + p.rows_per_slab - 1) / p.rows_per_slab);
  if (p.slabs < 1) p.slabs = 1;
  p.part_len = variant == kIso ? 2 + D : variant == kDiag ? 2 + 2 * D : 1 + D + D * D;
  return p;
}

}  // namespace

size_t general_workspace_bytes(int variant, int64_t N, int K, int D) {
  GeneralPlan p = plan_general(variant, N, K, D);
  WsCarve w(nullptr);
  w.take<int>(64);                                     // device status word (stays 0)
  w.take<float>(K);                                    // cst
  w.take<float>(variant == kDiag ? (size_t)K * D : K); // inv
  w.take<float>((size_t)p.slabs * K * p.part_len);     // partials
  return w.used + 256;
}

cudaError_t general_estep(int variant, const EstepArgs& a) {
  const int64_t N = a.N;
  const int K = a.K, D = a.D;
  GeneralPlan p = plan_general(variant, N, K, D);
  WsCarve w(a.ws);
  int* status = w.take<int>(64);  // the workspace's first word: no device-side failure here
  float* cst = w.take<float>(K);
  float* inv = w.take<float>(variant == kDiag ? (size_t)K * D : K);
  float* part = w.take<float>((size_t)p.slabs * K * p.part_len);
  cudaStream_t st = a.stream;

  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), st);
  if (e != cudaSuccess) return e;
  prep_kernel<<<(K + 127) / 128, 128, 0, st>>>(variant, a.cov, a.lpi, K, D, cst, inv);
  const unsigned row_blocks = (unsigned)((N + BR - 1) / BR);
  with_xtype(a.xtype, [&](auto tx) {
    using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
    const TX* X = a.x<TX>();
    if (variant != kFull) {
      const bool diag = variant == kDiag;
      if (diag)
        lse_kernel<true, TX><<<row_blocks, kThreads, 0, st>>>(X, a.sxn, a.sxd, a.mu, a.smk,
                                                              a.smd, inv, cst, N, K, D, a.logZ);
      else
        lse_kernel<false, TX><<<row_blocks, kThreads, 0, st>>>(X, a.sxn, a.sxd, a.mu, a.smk,
                                                               a.smd, inv, cst, N, K, D, a.logZ);
      const size_t dyn = ((size_t)3 * DC * (BR + PAD) + (size_t)3 * BR * (BC + PAD) +
                          (size_t)BC * D * (diag ? 2 : 1)) * sizeof(float);
      dim3 grid((K + BC - 1) / BC, p.slabs);
      profile_mark(false, st);
      if (diag) {
        ensure_dynamic_smem(reinterpret_cast<const void*>(stats_kernel<true, TX>), dyn);
        stats_kernel<true, TX><<<grid, kThreads, dyn, st>>>(X, a.sxn, a.sxd, a.mu, a.smk, a.smd,
                                                            inv, cst, N, K, D, a.logZ,
                                                            p.rows_per_slab, p.part_len, part);
      } else {
        ensure_dynamic_smem(reinterpret_cast<const void*>(stats_kernel<false, TX>), dyn);
        stats_kernel<false, TX><<<grid, kThreads, dyn, st>>>(X, a.sxn, a.sxd, a.mu, a.smk,
                                                             a.smd, inv, cst, N, K, D, a.logZ,
                                                             p.rows_per_slab, p.part_len, part);
      }
    } else {
      const size_t dyn = ((size_t)D * D + 2 * (size_t)BR * (D + 1)) * sizeof(float);
      ensure_dynamic_smem(reinterpret_cast<const void*>(full_lse_kernel<TX>), dyn);
      full_lse_kernel<TX><<<row_blocks, kThreads, dyn, st>>>(X, a.sxn, a.sxd, a.mu, a.smk, a.smd,
                                                             a.cov, cst, N, K, D, a.logZ);
      dim3 grid(K, p.slabs);
      profile_mark(false, st);
      if (D <= 64) {
        ensure_dynamic_smem(reinterpret_cast<const void*>(full_stats_kernel<4, TX>), dyn);
        full_stats_kernel<4, TX><<<grid, kThreads, dyn, st>>>(X, a.sxn, a.sxd, a.mu, a.smk,
                                                              a.smd, a.cov, cst, N, K, D, a.logZ,
                                                              p.rows_per_slab, p.part_len, part);
      } else {
        ensure_dynamic_smem(reinterpret_cast<const void*>(full_stats_kernel<8, TX>), dyn);
        full_stats_kernel<8, TX><<<grid, kThreads, dyn, st>>>(X, a.sxn, a.sxd, a.mu, a.smk,
                                                              a.smd, a.cov, cst, N, K, D, a.logZ,
                                                              p.rows_per_slab, p.part_len, part);
      }
    }
    return 0;
  });
  profile_mark(true, st);
  const int64_t total = (int64_t)K * p.part_len;
  const int rblocks = (int)std::min<int64_t>((total + 255) / 256, 8 * num_sms());
  reduce_kernel<<<rblocks, 256, 0, st>>>(variant, part, p.slabs, K, D, p.part_len, a.mu, a.smk,
                                         a.smd, a.Nk, a.mu_acc, a.sig,
                                         (a.flags & 1u) ? 1 : 0);
  count_launches(4);
  return cudaGetLastError();
}

}  // namespace fgmm
