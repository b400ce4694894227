// extern "C" entry points of libflashgmm_sm100.so (declared in
// include/flashgmm.h): argument validation, workspace checks, device check
// and the choice between the tensor-core kernels and the general kernels.
#include <stdio.h>

#include <atomic>
#include <map>
#include <mutex>
#include <string>

#include "../../include/flashgmm.h"
#include <algorithm>

#include "fgmm_internal.cuh"

namespace fgmm {
namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

// Compute capability check, cached per device (the library is built for
// sm_100a only and its kernels cannot run elsewhere).
int check_device(std::string* why) {
  static std::mutex mu;
  static int cc_cache[64] = {0};  // 0 unknown, >0 major*10+minor
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *why = std::string("cudaGetDevice failed: ") + cudaGetErrorString(e);
    return FGMM_ERR_CUDA;
  }
  int cc = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64) cc = cc_cache[dev];
  }
  if (cc == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cc = major * 10 + minor;
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64) cc_cache[dev] = cc;
  }
  if (cc != 100) {
    char buf[128];
    snprintf(buf, sizeof buf, "device %d has compute capability %d.%d; this library is built for sm_100a",
             dev, cc / 10, cc % 10);
    *why = buf;
    return FGMM_ERR_DEVICE;
  }
  return FGMM_OK;
}

__global__ void zero_outputs(int64_t K, int64_t D, int64_t sig_len, float* Nk, float* mu_acc,
                             float* sig) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < K * D + K + sig_len;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (i < K) Nk[i] = 0.f;
    else if (i < K + K * D) mu_acc[i - K] = 0.f;
    else sig[i - K - K * D] = 0.f;
  }
}

int64_t sig_len(int variant, int K, int D) {
  return variant == kIso ? K : variant == kDiag ? (int64_t)K * D : (int64_t)K * D * D;
}

int run_estep(int variant, EstepArgs a) {
  g_last_error.clear();
  const char* name = variant == kIso ? "fgmm_estep_iso"
                     : variant == kDiag ? "fgmm_estep_diag" : "fgmm_estep_full";
  char buf[256];
  if (a.N < 0 || a.K < 1 || a.D < 1) {
    snprintf(buf, sizeof buf, "%s: invalid shape N=%lld K=%d D=%d", name, (long long)a.N, a.K, a.D);
    return fail(FGMM_ERR_ARG, buf);
  }
  if (!a.mu || !a.cov || !a.lpi || !a.Nk || !a.mu_acc || !a.sig || (a.N > 0 && (!a.X || !a.logZ))) {
    snprintf(buf, sizeof buf, "%s: null pointer argument", name);
    return fail(FGMM_ERR_ARG, buf);
  }
  const int maxD = variant == kFull ? kGeneralMaxDFull : kGeneralMaxD;
  if (a.D > maxD) {
    snprintf(buf, sizeof buf, "%s: D=%d exceeds the supported maximum %d", name, a.D, maxD);
    return fail(FGMM_ERR_UNSUPPORTED, buf);
  }
  std::string why;
  int dc = check_device(&why);
  if (dc != FGMM_OK) return fail(dc, std::string(name) + ": " + why);

  if (a.N == 0) {  // no rows: statistics are zero (or unchanged when accumulating)
    if (!(a.flags & FGMM_FLAG_ACCUMULATE)) {
      zero_outputs<<<64, 256, 0, a.stream>>>(a.K, a.D, sig_len(variant, a.K, a.D), a.Nk,
                                            a.mu_acc, a.sig);
      count_launches(1);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(FGMM_ERR_CUDA, std::string(name) + ": " + cudaGetErrorString(e));
    return FGMM_OK;
  }

  const bool fast = !(a.flags & FGMM_FLAG_FORCE_GENERAL) && tc_supported(variant, a, nullptr);
  const size_t need = fast ? tc_workspace_bytes(variant, a.N, a.K, a.D)
                           : general_workspace_bytes(variant, a.N, a.K, a.D);
  if (need > 0 && (a.ws == nullptr || a.ws_bytes < need || (reinterpret_cast<uintptr_t>(a.ws) & 255))) {
    snprintf(buf, sizeof buf, "%s: workspace of %zu bytes (256-byte aligned) required, got %zu at %p",
             name, need, a.ws_bytes, a.ws);
    return fail(FGMM_ERR_WORKSPACE, buf);
  }
  cudaError_t e = fast ? tc_estep(variant, a) : general_estep(variant, a);
  if (e != cudaSuccess) return fail(FGMM_ERR_CUDA, std::string(name) + ": " + cudaGetErrorString(e));
  return FGMM_OK;
}

// ---------------------------------------------------------------------------
// Counter-based row generator.  Every value is a pure function of
// (seed, global row, feature): splitmix64 hashing, Box-Muller normals.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void gen_rows_kernel(float* __restrict__ X, const int64_t* __restrict__ row_ids,
                                int64_t row0, int64_t nrows, int D,
                                const float* __restrict__ centres, int K, uint64_t seed) {
  const int half = (D + 1) / 2;
  const int64_t total = nrows * half;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / half;
    const int p = (int)(e % half);
    const uint64_t n = (uint64_t)(row_ids ? row_ids[i] : row0 + i);
    const uint64_t hrow = mix64(seed ^ mix64(n));
    const int comp = (int)((hrow >> 11) % (uint64_t)K);
    const uint64_t h = mix64(hrow + 0x632BE59BD9B4E019ull * (uint64_t)(p + 1));
    const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = ((float)((h >> 8) & 0xFFFFFFu) + 0.5f) * (1.0f / 16777216.0f);
    const float rad = sqrtf(-2.0f * logf(u1));
    float s, c;
    sincospif(2.0f * u2, &s, &c);
    const int d0 = 2 * p;
    float* xr = X + i * (int64_t)D;
    xr[d0] = centres[(size_t)comp * D + d0] + rad * c;
    if (d0 + 1 < D) xr[d0 + 1] = centres[(size_t)comp * D + d0 + 1] + rad * s;
  }
}

}  // namespace

// Entry helpers for the other translation units' extern "C" functions.
int entry_fail(int code, const std::string& msg) { return fail(code, msg); }
int entry_check_device(std::string* why) { return check_device(why); }
int entry_run_estep(int variant, const EstepArgs& a) { return run_estep(variant, a); }

static std::atomic<uint64_t> g_launches{0};
static thread_local cudaEvent_t g_prof_start = nullptr, g_prof_stop = nullptr;

void count_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

void profile_mark(bool stop, cudaStream_t stream) {
  cudaEvent_t ev = stop ? g_prof_stop : g_prof_start;
  if (ev) cudaEventRecord(ev, stream);
}

static std::atomic<int> g_num_sms{0};
int num_sms() {
  int n = g_num_sms.load(std::memory_order_relaxed);
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_num_sms.store(n, std::memory_order_relaxed);
  }
  return n;
}

// The dynamic shared-memory limit of a kernel only ever grows (per kernel and
// device), so a launch that needs less never races with one that raised it.
cudaError_t ensure_dynamic_smem(const void* kernel, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> limit;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  size_t& cur = limit[{kernel, dev}];
  if (bytes <= cur) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) cur = bytes;
  return e;
}

cudaError_t generate_iso_rows(float* X, const int64_t* row_ids, int64_t row0, int64_t nrows,
                              int D, const float* centres, int K, uint64_t seed,
                              cudaStream_t stream) {
  if (nrows <= 0) return cudaSuccess;
  const int64_t total = nrows * ((D + 1) / 2);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 16 * num_sms());
  gen_rows_kernel<<<blocks, 256, 0, stream>>>(X, row_ids, row0, nrows, D, centres, K, seed);
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace fgmm

using fgmm::EstepArgs;

extern "C" {

int fgmm_version(void) { return 100; }

const char* fgmm_last_error(void) { return fgmm::g_last_error.c_str(); }

uint64_t fgmm_launch_count(void) { return fgmm::g_launches.load(std::memory_order_relaxed); }

void fgmm_set_profile_events(void* start_event, void* stop_event) {
  fgmm::g_prof_start = reinterpret_cast<cudaEvent_t>(start_event);
  fgmm::g_prof_stop = reinterpret_cast<cudaEvent_t>(stop_event);
}

size_t fgmm_workspace_bytes(int variant, int64_t N, int32_t K, int32_t D) {
  if (variant < 0 || variant > 2 || N < 0 || K < 1 || D < 1) return 0;
  size_t g = fgmm::general_workspace_bytes(variant, N, K, D);
  size_t t = fgmm::tc_workspace_bytes(variant, N, K, D);
  return g > t ? g : t;
}

#define FGMM_ESTEP_BODY(VARIANT)                                                       \
  EstepArgs a{X, x_stride_n, x_stride_d, mu, mu_stride_k, mu_stride_d, COV, log_pi, N, \
              K, D, logZ, Nk, mu_acc, SIG, workspace, workspace_bytes, flags,          \
              reinterpret_cast<cudaStream_t>(stream)};                                 \
  return fgmm::run_estep(VARIANT, a);

int fgmm_estep_iso(const float* X, int64_t x_stride_n, int64_t x_stride_d, const float* mu,
                   int64_t mu_stride_k, int64_t mu_stride_d, const float* log_sigma_sq,
                   const float* log_pi, int64_t N, int32_t K, int32_t D, float* logZ, float* Nk,
                   float* mu_acc, float* sig_acc, void* workspace, size_t workspace_bytes,
                   unsigned flags, void* stream) {
#define COV log_sigma_sq
#define SIG sig_acc
  FGMM_ESTEP_BODY(fgmm::kIso)
#undef COV
#undef SIG
}

int fgmm_estep_diag(const float* X, int64_t x_stride_n, int64_t x_stride_d, const float* mu,
                    int64_t mu_stride_k, int64_t mu_stride_d, const float* log_sigma_sq,
                    const float* log_pi, int64_t N, int32_t K, int32_t D, float* logZ,
                    float* Nk, float* mu_acc, float* sig_acc, void* workspace,
                    size_t workspace_bytes, unsigned flags, void* stream) {
#define COV log_sigma_sq
#define SIG sig_acc
  FGMM_ESTEP_BODY(fgmm::kDiag)
#undef COV
#undef SIG
}

int fgmm_estep_full(const float* X, int64_t x_stride_n, int64_t x_stride_d, const float* mu,
                    int64_t mu_stride_k, int64_t mu_stride_d, const float* prec_chol,
                    const float* log_pi, int64_t N, int32_t K, int32_t D, float* logZ,
                    float* Nk, float* mu_acc, float* sig_outer, void* workspace,
                    size_t workspace_bytes, unsigned flags, void* stream) {
#define COV prec_chol
#define SIG sig_outer
  FGMM_ESTEP_BODY(fgmm::kFull)
#undef COV
#undef SIG
}

int fgmm_estep_x(int variant, int x_type, const void* X, int64_t x_stride_n, int64_t x_stride_d,
                 const float* mu, int64_t mu_stride_k, int64_t mu_stride_d, const float* cov,
                 const float* log_pi, int64_t N, int32_t K, int32_t D, float* logZ, float* Nk,
                 float* mu_acc, float* sig, void* workspace, size_t workspace_bytes,
                 unsigned flags, void* stream) {
  fgmm::g_last_error.clear();
  if (variant < 0 || variant > 2)
    return fgmm::fail(FGMM_ERR_ARG, "fgmm_estep_x: unknown variant " + std::to_string(variant));
  if (x_type != FGMM_X_F32 && x_type != FGMM_X_BF16)
    return fgmm::fail(FGMM_ERR_ARG, "fgmm_estep_x: unknown x_type " + std::to_string(x_type));
  EstepArgs a{X, x_stride_n, x_stride_d, mu, mu_stride_k, mu_stride_d, cov, log_pi, N,
              K, D, logZ, Nk, mu_acc, sig, workspace, workspace_bytes, flags,
              reinterpret_cast<cudaStream_t>(stream)};
  a.xtype = x_type == FGMM_X_BF16 ? fgmm::kXBF16 : fgmm::kXF32;
  return fgmm::run_estep(variant, a);
}

int fgmm_generate_iso_rows(float* X, const int64_t* row_ids, int64_t row0, int64_t nrows,
                           int32_t D, const float* centres, int32_t K, uint64_t seed,
                           void* stream) {
  fgmm::g_last_error.clear();
  if (nrows < 0 || D < 1 || K < 1 || (nrows > 0 && (!X || !centres)))
    return fgmm::fail(FGMM_ERR_ARG, "fgmm_generate_iso_rows: invalid arguments");
  std::string why;
  int dc = fgmm::check_device(&why);
  if (dc != FGMM_OK) return fgmm::fail(dc, "fgmm_generate_iso_rows: " + why);
  cudaError_t e = fgmm::generate_iso_rows(X, row_ids, row0, nrows, D, centres, K, seed,
                                          reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fgmm::fail(FGMM_ERR_CUDA, std::string("fgmm_generate_iso_rows: ") + cudaGetErrorString(e));
  return FGMM_OK;
}

}  // extern "C"
