// Isotropic E-step kernel for K <= 1024 components and D <= 128 features
// (the reference's headline shape, flash_gmm.py:50-166 and
// flash_gmm_h100.py:85-243): one launch computes logZ and the per-cluster
// partial statistics, with the distance GEMM evaluated once per
// (row, component) pair.  Included by fgmm_tc.cu (namespace fgmm::{anon}),
// whose split, prep and reduce kernels it shares.
//
// Orientation: a CTA owns 128 components (the TMEM lanes); a cluster of
// C = ceil(K/128) CTAs covers all components and walks the same 128-row
// tiles.  W (fp16 hi/lo) is the resident TMEM A operand, so the distance
// MMAs read only the row tile from shared memory.
//
// Per 128-row tile j (S buffer b = j & 1), for each 32-row block and each
// quadrant of 32 components (one epilogue warp; lane = component):
//   MMA dist(j):  S[b] = W_lo X_hi + W_hi X_lo + W_hi X_hi   (24 MMAs, N = 128)
//   A   ll = S 2^(a+s_k) + c0' - ish |x-c|^2 (log2 units) for the block's 32
//       rows, read in the 16x256b fragment layout (4 components x 8 rows per
//       thread); per row the quadrant's max m and the fp32 sum of
//       p = 2^(ll - m) by in-thread max/add plus 3 shuffle rounds;
//   B   (lane = row; each of the block's four warps) the four quadrants'
//       pairs (shared memory) -> the CTA's (max, sum) per row, sent to the
//       cluster's CTAs (st.async; warp q serves peers q and q + 4); every
//       CTA's pair -> the row's log2-normaliser lz2 = M + log2 S;
//   C   rows where the quadrant's max is within 2^25 of lz2:
//       r = 2^(ll - lz2), split into fp16 hi/lo words and written to TMEM
//       over the block's own S columns (hi in the first 16, lo in the next
//       16); every other row's responsibilities are below 2^-25, which
//       rounds to zero in fp16, and are written as zeros; Nk and sum r ll
//       per component are per-thread sums (thread = component);
//   MMA stats(j): T += R^T X  (3 terms r_lo x_hi + r_hi x_lo + r_hi x_hi,
//       24 MMAs; A = R^T in TMEM, B = the row tile read MN-major).
// The selection in C is made for 32 rows at once (lane = row,
// vote.ballot), so the work follows the number of rows a quadrant takes part
// in: all of them for overlapping components, about one in 32 when each row
// belongs to one well separated component.  Up to four selected rows of a
// block are re-read with single-column TMEM loads issued together and the
// block's words written in one pass; more, with one 32-column load.  The
// results do not depend on the selection beyond the stated cut-offs.
//
// Both GEMMs carry 22-bit operands (fp16 hi/lo, exact power-of-two scaling):
// logZ is held to 1e-5 and the statistics to 1e-4 also where the rows of a
// component nearly cancel.  The MMA warp issues dist(j+1) and stats(j-1)
// while the epilogue works on tile j: S is double-buffered and the tensor
// pipe executes in issue order, so dist(j+2) (into S[b]) follows stats(j),
// which read R^T from S[b].
//
// TMEM (512 columns): W hi [0,64) lo [64,128) | T [128,256) | S0 [256,384) |
// S1 [384,512).  Warps 0-15: epilogue (warp w: lane quadrant w & 3, row
// block w >> 2); warp 16 loads row tiles (one bulk copy per stage); warp 17
// issues MMAs.  Every wait is bounded; a timeout sets the error word and the
// kernel leaves its loops (the reduction then writes NaN).

constexpr int kIsoEpiWarps = 16;
constexpr int kIsoWarps = kIsoEpiWarps + 2;      // 18
constexpr int kIsoThreads = kIsoWarps * 32;      // 576
constexpr int kIsoLoadWarp = kIsoEpiWarps;       // 16
constexpr int kIsoMmaWarp = kIsoEpiWarps + 1;    // 17
constexpr int kIsoStages = 3;
constexpr int kIsoRows = 128;
constexpr int kIsoMaxD = 128;
constexpr int kIsoCluster = 8;
constexpr uint32_t kIsoColW = 0, kIsoColT = 128, kIsoColS = 256;
constexpr float kRespCut = 25.f;  // C: quadrant max below lz2 - 25: r = 0

struct __align__(8) IsoCtl {
  uint64_t xfull[kIsoStages];
  uint64_t xempty[kIsoStages];
  uint64_t s_full[2];
  uint64_t r_full[2];
  uint64_t t_done;
  uint64_t xchg_full[2][4];  // [tile parity][row block]
  uint64_t e_bar[4];         // [row block]: phase A done, one arrival per quadrant warp
  uint64_t e_end;
  uint32_t tmem_base;
  volatile int abort_flag;
};

// Shared-memory carve-up (offsets from the 1024-aligned base).
struct IsoSmem {
  static constexpr int kStageMax = 2 * 2 * kIsoRows * 128;           // 64 KB
  static constexpr int kXs = 0;
  static constexpr int kXsq = kXs + kIsoStages * kStageMax;          // [NS][128] f32
  // per tile parity, row block, quadrant and row: the quadrant's max and its
  // sum of 2^(ll - max) (f32)
  static constexpr int kQMax = kXsq + kIsoStages * kIsoRows * 4;     // [2][4 blk][4 q][32]
  static constexpr int kQSum = kQMax + 2 * 16 * 32 * 4;              // [2][4 blk][4 q][32]
  static constexpr int kFin = kQSum + 2 * 16 * 32 * 4;               // [8][128] f32
  static constexpr int kXchg = kFin + 8 * kComps * 4;                // [2][8][128] f2
  static constexpr int kCtl = kXchg + 2 * kIsoCluster * kIsoRows * 8;
  static constexpr int kBytes = kCtl + (int)sizeof(IsoCtl);
  static constexpr size_t kDynamic = 1024 + (size_t)kBytes;          // alignment slack
};
static_assert(IsoSmem::kDynamic <= 232448, "shared memory budget");

__device__ __forceinline__ bool iso_wait(uint64_t* b, uint32_t parity, IsoCtl* ctl, int* err,
                                         int code) {
  return mbar_wait_flag<false>(b, parity, &ctl->abort_flag, err, code);
}

__global__ void __launch_bounds__(kIsoThreads, 1) tc_iso_kernel(const TcParams p) {
  constexpr int NS = kIsoStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int stage_bytes = 2 * p.nch * kIsoRows * 128;  // hi + lo
  uint8_t* xs = smem + IsoSmem::kXs;
  float* xsq = reinterpret_cast<float*>(smem + IsoSmem::kXsq);
  float* qmax = reinterpret_cast<float*>(smem + IsoSmem::kQMax);
  float* qsum = reinterpret_cast<float*>(smem + IsoSmem::kQSum);
  float* fin = reinterpret_cast<float*>(smem + IsoSmem::kFin);
  float2* xchg = reinterpret_cast<float2*>(smem + IsoSmem::kXchg);  // [slot][CTA][row]
  IsoCtl* ctl = reinterpret_cast<IsoCtl*>(smem + IsoSmem::kCtl);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int cluster_id = blockIdx.x / p.C;
  const int num_clusters = gridDim.x / p.C;
  const int ntiles = (p.num_tiles - cluster_id + num_clusters - 1) / num_clusters;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&ctl->xfull[s], 1);   // loader's arrive.expect_tx + bulk-copy bytes
      mbar_init(&ctl->xempty[s], 1);  // commit after the tile's statistics MMAs
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->s_full[b], 1);             // commit after the distance MMAs
      mbar_init(&ctl->r_full[b], kIsoEpiWarps);  // every epilogue warp wrote its R^T
    }
    mbar_init(&ctl->t_done, 1);
    for (int cb = 0; cb < 4; ++cb) {
      mbar_init(&ctl->xchg_full[0][cb], 1);  // local arrive.expect_tx + peers' st.async bytes
      mbar_init(&ctl->xchg_full[1][cb], 1);
      mbar_init(&ctl->e_bar[cb], 4);
    }
    mbar_init(&ctl->e_end, kIsoEpiWarps);
    ctl->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {  // all 512 TMEM columns (one CTA per SM)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(&ctl->tmem_base))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  const int q = warp & 3, cb = (warp >> 2) & 3;  // epilogue: lane quadrant, row block
  const int kl = q * 32 + lane;                  // local component (TMEM lane)
  const int kg = (int)rank * kComps + kl;        // global component
  float4 kc = make_float4(-1e30f, 0.f, -1e30f, 0.f);
  if (warp < kIsoEpiWarps) kc = p.consts[kg];
  const int xa = x_scale_exp<false>(__int_as_float(*p.xscale));  // x' = (x - c) 2^-xa

  // zero the stages once: padding features of a partial last chunk stay 0
  for (int i = threadIdx.x; i < NS * stage_bytes / 16; i += kIsoThreads)
    reinterpret_cast<uint4*>(xs)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  // W rows into TMEM (A operand of the distance GEMM), lane = component
  if (warp < 4) {
    const uint4* wh = reinterpret_cast<const uint4*>(p.Whi + (size_t)kg * p.nfeat);
    const uint4* wl = reinterpret_cast<const uint4*>(p.Wlo + (size_t)kg * p.nfeat);
    const uint32_t lb = (uint32_t)(q * 32) << 16;
    for (int s = 0; s < p.nfeat / 16; ++s) {
      uint32_t v[8];
      uint4 a = wh[2 * s], c = wh[2 * s + 1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
      tmem_st8(tmem + lb + kIsoColW + 8 * s, v);
      a = wl[2 * s];
      c = wl[2 * s + 1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
      tmem_st8(tmem + lb + kIsoColW + 64 + 8 * s, v);
    }
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // peers' barriers are initialised before any remote arrive
  tc_fence_after();

  if (warp == kIsoMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (waits, addresses: warp-uniform values);
    // one elected lane issues each batch of MMAs.  Descriptors are formed
    // once per stage and advanced by constant offsets, so an MMA costs about
    // one integer add to set up: the issuing warp shares its sub-partition
    // with four epilogue warps, and a longer setup left the tensor pipe idle
    // between MMAs.
    const uint32_t id_dist = idesc_f16(kIsoRows, false);
    const uint32_t id_stat = idesc_f16(64 * p.nch, true);
    const int ksd = p.nfeat / 16;
    const uint32_t lo_off = (uint32_t)(p.nch * kIsoRows * 128);
    const uint32_t xs0 = smem_u32(xs);
    constexpr uint32_t kChunkBytes = kIsoRows * 128;  // one 64-feature chunk of a stage
    auto issue_stats = [&](int jj) {
      const uint32_t xhi = xs0 + (uint32_t)((jj % NS) * stage_bytes);
      const uint32_t dhi = desc_lo_mnmajor(xhi, kChunkBytes);
      const uint32_t dlo = desc_lo_mnmajor(xhi + lo_off, kChunkBytes);
      const uint32_t rcol = tmem + kIsoColS + 128u * (uint32_t)(jj & 1);
      const uint32_t tcol = tmem + kIsoColT;
      if (elect_one()) {
        // terms r_lo x_hi, r_hi x_lo, r_hi x_hi; K-step s = rows 16s..16s+15 =
        // row block s/2, columns 8 (s & 1) of its hi (+0) / lo (+16) words;
        // B advances 16 rows = 2048 bytes per K-step
#pragma unroll
        for (int t = 0; t < 3; ++t) {
          const uint32_t aoff = t == 0 ? 16u : 0u;
          const uint32_t bd = t == 1 ? dlo : dhi;
#pragma unroll
          for (int s = 0; s < kIsoRows / 16; ++s)
            mma_ts2(tcol, rcol + 32u * (uint32_t)(s >> 1) + 8u * (uint32_t)(s & 1) + aoff,
                    bd + (uint32_t)(s * (2048 >> 4)), kDescHi, id_stat,
                    (jj == 0 && t == 0 && s == 0) ? 0u : 1u);
        }
        tc_commit(&ctl->xempty[jj % NS]);
      }
      __syncwarp();
    };
    // warp-uniform outcome of a bounded wait (elect_one needs every lane)
    auto wait_all = [&](uint64_t* bar, uint32_t parity, int code) {
      return __all_sync(0xffffffffu, iso_wait(bar, parity, ctl, p.err, code));
    };
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % NS;
      if (!wait_all(&ctl->xfull[st], (j / NS) & 1, 1)) { ok = false; break; }
      tc_fence_after();
      const uint32_t xhi = xs0 + (uint32_t)(st * stage_bytes);
      const uint32_t dhi = desc_lo_kmajor(xhi), dlo = desc_lo_kmajor(xhi + lo_off);
      const uint32_t scol = tmem + kIsoColS + 128u * (uint32_t)(j & 1);
      if (elect_one()) {
        // terms W_lo x_hi, W_hi x_lo, W_hi x_hi (smallest magnitudes first);
        // K-step s: chunk s/4 (kChunkBytes apart), 32 bytes within the row
#pragma unroll
        for (int t = 0; t < 3; ++t) {
          const uint32_t acol = tmem + kIsoColW + (t == 0 ? 64u : 0u);
          const uint32_t bd = t == 1 ? dlo : dhi;
#pragma unroll
          for (int s = 0; s < kIsoMaxD / 16; ++s)
            if (s < ksd)
              mma_ts2(scol, acol + 8u * (uint32_t)s,
                      bd + (uint32_t)(((s >> 2) * kChunkBytes + (s & 3) * 32) >> 4), kDescHi,
                      id_dist, (t == 0 && s == 0) ? 0u : 1u);
        }
        tc_commit(&ctl->s_full[j & 1]);
      }
      __syncwarp();
      if (j >= 1) {
        if (!wait_all(&ctl->r_full[(j - 1) & 1], ((j - 1) >> 1) & 1, 4)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_stats(j - 1);
      }
    }
    if (ok && ntiles >= 1 && wait_all(&ctl->r_full[(ntiles - 1) & 1], ((ntiles - 1) >> 1) & 1, 4)) {
      tc_fence_after();
      issue_stats(ntiles - 1);
      if (elect_one()) tc_commit(&ctl->t_done);
      __syncwarp();
    }
  } else if (warp == kIsoLoadWarp) {
    // ------------------------------------------------------------ row-tile loader
    if (lane == 0) {
      const uint32_t tx = (uint32_t)stage_bytes + kIsoRows * 4u;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % NS;
        const int64_t tile = cluster_id + (int64_t)j * num_clusters;
        if (!iso_wait(&ctl->xempty[st], ((j / NS) & 1) ^ 1, ctl, p.err, 8)) break;
        mbar_arrive_expect_tx(&ctl->xfull[st], tx);
        bulk_g2s(smem_u32(xs + st * stage_bytes), p.xsplit + tile * stage_bytes,
                 (uint32_t)stage_bytes, &ctl->xfull[st]);
        bulk_g2s(smem_u32(xsq + st * kIsoRows), p.xsq + tile * kIsoRows, kIsoRows * 4u,
                 &ctl->xfull[st]);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- epilogue
    const float c0p = kc.x, ish = kc.y, c0 = kc.z;
    const float sck = ldexpf(1.0f, xa + (int)kc.w);  // ll = S' 2^(a + s_k) + ...
    // Equal variances: every component's ll has the same row term
    // -ish |x-c|^2, which a row's log-sum-exp carries through unchanged, so
    // the reductions run on ll' = S' 2^(a+s_k) + c0' (one FFMA per pair) and
    // the term is applied once per row (lz2 = lz2' - ish |x-c|^2).
    const bool uni = p.nonuniform != nullptr && *p.nonuniform == 0;
    const float ish_row = uni ? p.consts[0].y : 0.f;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float nk_acc = 0.f, rll_acc = 0.f;
    // Phase A reads S in the 16x256b fragment layout: thread t holds the
    // components (quadrant lanes) t/4 + 8u, u = 0..3, at the block's rows
    // 8j + 2(t%4) + e, j = 0..3, e = 0..1; their constants:
    float ac0[4], asck[4], aish[4];
    if (warp < kIsoEpiWarps) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 c4 = p.consts[(int)rank * kComps + q * 32 + (lane >> 2) + 8 * u];
        ac0[u] = c4.x;
        aish[u] = c4.y;
        asck[u] = ldexpf(1.0f, xa + (int)c4.w);
      }
    }
    const int rsub = 2 * (lane & 3);  // this thread's rows: 8j + rsub + e
    // Expanded-form accuracy: the distance comes out of an fp32 tensor-core
    // accumulation whose error grows with ish |x - c| |mu_k - c| (up to ~14
    // units of 2^-23 of it, measured), while logZ is held to 1e-5 of |logZ|.
    // Pairs with r >= 2^-8 where 32 x 2^-23 of that magnitude exceeds the
    // tolerance are listed for an exact recomputation of their distance from
    // the inputs (tc_refine_iso_kernel), which corrects logZ.
    const float mck = (p.refine != nullptr && warp < kIsoEpiWarps) ? p.mc[kg] : 0.f;
    const float cmax = redux_max(ish * mck) * 3.814697265625e-06f;  // ish, mck >= 0
    const float cgate = cmax * cmax;
    auto sync_block = [&](int j, int code) -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->e_bar[cb]);
      return iso_wait(&ctl->e_bar[cb], j & 1, ctl, p.err, code);
    };
    // peers' pair slots for this lane's row and the barrier words, per slot
    const int xrow = 32 * cb + lane;
    for (int j = 0; j < ntiles; ++j) {
      const int b = j & 1, st = j % NS, slot = j & 1;
      const int64_t row0 = (int64_t)(cluster_id + (int64_t)j * num_clusters) * kIsoRows;
      const uint32_t scol = tmem + lane_base + kIsoColS + 128u * (uint32_t)b + 32u * (uint32_t)cb;
      const float* xq = xsq + st * kIsoRows + 32 * cb;
      float* qm = qmax + (slot * 4 + cb) * 128;     // [4 q][32 rows] of this row block
      float* qs = qsum + (slot * 4 + cb) * 128;
      if (!iso_wait(&ctl->s_full[b], (j >> 1) & 1, ctl, p.err, 16)) break;
      if (!iso_wait(&ctl->xfull[st], (j / NS) & 1, ctl, p.err, 4096)) break;
      tc_fence_after();
      // ---- A: per row, the quadrant's max m and the sum of p = 2^(ll - m)
      // over the quadrant's 32 components.  In the 16x256b layout each row's
      // 32 values sit on the 8 threads sharing t % 4, four per thread: the
      // max is 3 in-thread max + a 3-step xor butterfly, the sum 3 in-thread
      // adds + a 3-round transpose-reduce, after which thread t holds the row
      // 8 (t/8) + 2 (t%4) + (t/4)%2 and records its (max, sum).
      {
        uint32_t v[32];
        tmem_ld16x256_x4(scol, v);
        tmem_ld16x256_x4(scol + (16u << 16), v + 16);
        tmem_wait_ld();
        float mr[8], sr[8];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          float xv[2] = {0.f, 0.f};
          if (!uni) {
            const float2 x2 = *reinterpret_cast<const float2*>(xq + 8 * jj + rsub);
            xv[0] = x2.x;
            xv[1] = x2.y;
          }
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float ll[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float base = uni ? ac0[u] : fmaf(-aish[u], xv[e], ac0[u]);
              ll[u] = fmaf(__uint_as_float(v[16 * (u >> 1) + 4 * jj + 2 * (u & 1) + e]), asck[u],
                           base);
            }
            float m = fmaxf(fmaxf(ll[0], ll[1]), fmaxf(ll[2], ll[3]));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
            mr[2 * jj + e] = m;
            sr[2 * jj + e] = (ex2(ll[0] - m) + ex2(ll[1] - m)) + (ex2(ll[2] - m) + ex2(ll[3] - m));
          }
        }
        // transpose-reduce of the 8 row sums over lane bits 4, 3, 2 (row-index
        // bits 2, 1, 0); the max (equal on the 8 threads) is selected alongside
#pragma unroll
        for (int h = 4, msk = 16; h >= 1; h >>= 1, msk >>= 1) {
          const bool up = (lane & msk) != 0;
#pragma unroll
          for (int i = 0; i < h; ++i) {
            const float send = up ? sr[i] : sr[i + h];
            const float keep = up ? sr[i + h] : sr[i];
            sr[i] = keep + __shfl_xor_sync(0xffffffffu, send, msk);
            mr[i] = up ? mr[i + h] : mr[i];
          }
        }
        const int ri = (lane >> 2) & 7;  // row index 2j + e held now
        const int row = 8 * (ri >> 1) + rsub + (ri & 1);
        qm[q * 32 + row] = mr[0];
        qs[q * 32 + row] = sr[0];
      }
      if (!sync_block(j, 256)) break;
      // ---- B (lane = row of the block; each of the block's four warps does
      // this for all 32 rows, so no second block-wide sync is needed): the
      // CTA's (max, sum) from the four quadrants, sent to peers q and q + 4;
      // then every CTA's pair -> the row's log2-normaliser lz2
      float mq, lz;
      {
        float mqq[4], sqq[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          mqq[u] = qm[u * 32 + lane];
          sqq[u] = qs[u * 32 + lane];
        }
        mq = q == 0 ? mqq[0] : q == 1 ? mqq[1] : q == 2 ? mqq[2] : mqq[3];
        const float M = fmaxf(fmaxf(mqq[0], mqq[1]), fmaxf(mqq[2], mqq[3]));
        float L = 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) L = fmaf(sqq[u], ex2(mqq[u] - M), L);
        float2* xb = xchg + slot * kIsoCluster * kIsoRows;
        const uint32_t my_slot = smem_u32(&xb[rank * kIsoRows + xrow]);
        const uint32_t my_bar = smem_u32(&ctl->xchg_full[slot][cb]);
        if (q == 0 && lane == 0)
          mbar_arrive_expect_tx(&ctl->xchg_full[slot][cb], (uint32_t)(p.C * 32 * 8));
#pragma unroll
        for (int jj = 0; jj < 2; ++jj)
          if (q + 4 * jj < p.C)
            st_async_f2(map_to_cta(my_slot, q + 4 * jj), M, L, map_to_cta(my_bar, q + 4 * jj));
        if (!mbar_wait_flag<true>(&ctl->xchg_full[slot][cb], (j >> 1) & 1, &ctl->abort_flag,
                                  p.err, 32))
          break;
        float2 e[kIsoCluster];
        float GM = -3e38f;
#pragma unroll
        for (int c = 0; c < kIsoCluster; ++c) {
          e[c] = c < p.C ? xb[c * kIsoRows + xrow] : make_float2(-3e38f, 0.f);
          GM = fmaxf(GM, e[c].x);
        }
        float GL = 0.f;
#pragma unroll
        for (int c = 0; c < kIsoCluster; ++c)
          if (c < p.C) GL = fmaf(e[c].y, ex2(e[c].x - GM), GL);
        const float lz2 = GM + lg2(GL);  // in the reductions' units (ll' when uni)
        const bool valid = row0 + xrow < p.N;
        if (valid && rank == 0 && q == 0)
          p.logZ[row0 + xrow] = fmaf(-ish_row, xq[lane], lz2) * 0.6931471805599453f;
        lz = valid ? lz2 : __int_as_float(0x7f800000);  // +inf: r = 0
      }

      // ---- C: responsibilities of the rows this quadrant takes part in;
      // R^T (fp16 hi | lo) over the block's own S columns, zeros elsewhere
      {
        const uint32_t need = __ballot_sync(0xffffffffu, mq >= lz - kRespCut);
        const uint32_t pairs = (need | (need >> 1)) & 0x55555555u;
        float nk_t = 0.f, rll_t = 0.f;
        // Pairs for the exact refinement: r >= 2^-8 and
        // 32 x 2^-23 ish |x - c| |mu_k - c| > 1e-5 max(1, |logZ|) (log2 units);
        // only rows whose |x - c| / max(1, |logZ|) times the warp's largest
        // ish |mu_k - c| could pass are scanned (on C2 about one in a hundred)
        if (p.refine != nullptr) {
          const float xl = xq[lane];  // lane = row; squared form of the test, no sqrt
          const float tl = 1e-5f * fmaxf(1.44269504f, fabsf(uni ? fmaf(-ish_row, xl, lz) : lz));
          const uint32_t cand = __ballot_sync(0xffffffffu, xl * cgate > tl * tl);
          if (cand & need) {
            for (uint32_t nm = cand & need; nm != 0u; nm &= nm - 1u) {
              const int i = __ffs(nm) - 1;
              const float sv1 = __uint_as_float(tmem_ld1(scol + (uint32_t)i));
              tmem_wait_ld();
              const float x = xq[i];
              const float lzi = __shfl_sync(0xffffffffu, lz, i);
              const float ll = uni ? fmaf(sv1, sck, c0p) : fmaf(sv1, sck, fmaf(-ish, x, c0p));
              const float r = ex2(ll - lzi);
              const float lzt = uni ? fmaf(-ish_row, x, lzi) : lzi;
              const float tt = 1e-5f * fmaxf(1.44269504f, fabsf(lzt));
              const float bk = ish * mck * 3.814697265625e-06f;
              if (r >= 0.00390625f && x * bk * bk > tt * tt) {
                const int at = atomicAdd(p.refine_count, 1);
                if (at < p.refine_cap)
                  p.refine[at] = make_int4(p.row_base + (int)row0 + 32 * cb + i, kg,
                                           __float_as_int(r),
                                           __float_as_int(uni ? fmaf(-ish, x, ll) : ll));
              }
            }
          }
        }
        // r of row i from this lane's distance s (ll in the reductions'
        // units; sum r ll in true units)
        auto resp = [&](int i, float s) {
          const float x = xq[i];
          const float ll = uni ? fmaf(s, sck, c0p) : fmaf(s, sck, fmaf(-ish, x, c0p));
          const float r = ex2(ll - __shfl_sync(0xffffffffu, lz, i));
          nk_t += r;
          rll_t = fmaf(r, uni ? fmaf(-ish, x, ll) : ll, rll_t);
          return r;
        };
        if (__popc(pairs) <= 2) {
          // at most two column pairs: read their distances, zero the block's
          // words (R^T replaces S in place), then write the pairs' words
          int i0[2];
          uint32_t v[4];
          uint32_t pm = pairs;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            i0[u] = pm ? __ffs(pm) - 1 : -1;
            pm &= pm - 1;
            const uint32_t c = i0[u] >= 0 ? (uint32_t)i0[u] : 0u;
            v[2 * u] = tmem_ld1(scol + c);
            v[2 * u + 1] = tmem_ld1(scol + c + 1u);
          }
          tmem_wait_ld();
          uint32_t h[2] = {0u, 0u}, l[2] = {0u, 0u};
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            if (i0[u] < 0) continue;
            const int i = i0[u];
            const float r0 = ((need >> i) & 1u) ? resp(i, __uint_as_float(v[2 * u])) : 0.f;
            const float r1 =
                ((need >> (i + 1)) & 1u) ? resp(i + 1, __uint_as_float(v[2 * u + 1])) : 0.f;
            split2(r0, r1, h[u], l[u]);
          }
          // the block's 16 hi and 16 lo words in one pass: the (at most two)
          // computed column pairs, zeros elsewhere
          const int c0 = i0[0] >= 0 ? (i0[0] >> 1) : -1;
          const int c1 = i0[1] >= 0 ? (i0[1] >> 1) : -1;
          uint32_t hv[16], lv[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            hv[c] = c == c0 ? h[0] : (c == c1 ? h[1] : 0u);
            lv[c] = c == c0 ? l[0] : (c == c1 ? l[1] : 0u);
          }
          tmem_st16(scol, hv);
          tmem_st16(scol + 16, lv);
        } else {
          uint32_t sv[32];
          tmem_ld32(scol, sv);
          tmem_wait_ld();
          uint32_t hv[16], lv[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float r0 = ((need >> (2 * c)) & 1u) ? resp(2 * c, __uint_as_float(sv[2 * c])) : 0.f;
            const float r1 =
                ((need >> (2 * c + 1)) & 1u) ? resp(2 * c + 1, __uint_as_float(sv[2 * c + 1])) : 0.f;
            split2(r0, r1, hv[c], lv[c]);
          }
          tmem_st16(scol, hv);
          tmem_st16(scol + 16, lv);
        }
        nk_acc += nk_t;
        rll_acc += rll_t;
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->r_full[b]);
    }

    // End: statistics accumulator -> per-cluster partials {Nk, sig, T 2^a}.
    fin[cb * kComps + kl] = nk_acc;
    fin[(4 + cb) * kComps + kl] = rll_acc;
    __syncwarp();
    if (lane == 0) mbar_arrive(&ctl->e_end);
    const bool ok = !ctl->abort_flag && ntiles >= 1 &&
                    iso_wait(&ctl->e_end, 0, ctl, p.err, 1024) &&
                    iso_wait(&ctl->t_done, 0, ctl, p.err, 128);
    float* out = p.part + ((size_t)cluster_id * p.C * kComps + kg) * p.plen;
    if (ok) {
      tc_fence_after();
      if (32 * cb < 64 * p.nch) {
        uint32_t tv[32];
        tmem_ld32(tmem + lane_base + kIsoColT + 32 * cb, tv);
        tmem_wait_ld();
        for (int i = 0; i < 32; ++i) {
          const int f = 32 * cb + i;
          if (f < p.D) out[2 + f] = ldexpf(__uint_as_float(tv[i]), xa);  // T = T' 2^a
        }
      }
      if (cb == 0) {
        const float nk = fin[kl] + fin[kComps + kl] + fin[2 * kComps + kl] + fin[3 * kComps + kl];
        const float rl = fin[4 * kComps + kl] + fin[5 * kComps + kl] + fin[6 * kComps + kl] +
                         fin[7 * kComps + kl];
        out[0] = nk;
        out[1] = ish > 0.f ? (c0 * nk - rl) / ish : 0.f;
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
