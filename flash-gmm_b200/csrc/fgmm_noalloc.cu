// fgmm_estep_iso_noalloc: the isotropic E-step with its scratch taken from a
// fixed-size device array that this library owns, instead of a workspace the
// caller passes in.
//
// Who needs it: callers that hold no device allocator they may use at the
// call site -- a host runtime whose device memory is owned by another pool
// (a JVM or Go process binding the C ABI next to a framework's caching
// allocator), or a latency-critical loop that must not call cudaMalloc,
// which can synchronise the device.  Such a caller gets the same kernels
// and the same results as fgmm_estep_iso, with nothing allocated per call.
//
// Limits and rules:
//  * The scratch is FGMM_NOALLOC_SCRATCH_BYTES (64 MiB) per device; a shape
//    whose workspace (what fgmm_estep_iso would need on the path it takes)
//    is larger is rejected with FGMM_ERR_WORKSPACE before anything runs.
//  * Nothing in the scratch has to start at zero: every kernel of the path
//    writes the scratch words it reads earlier in the same call (the fast
//    path clears its error/scale words with cudaMemsetAsync first).
//  * One array per device, shared by every call on that device: two calls
//    that can overlap in time (different streams, or different host threads
//    without ordering between them) race on it.  Order them on one stream.
//  * The first call on each device does the set-up: with that device current
//    it asks the runtime for the array's device address (under the runtime's
//    default lazy module loading this is what loads this file's module and
//    with it the array) and caches the pointer.  Make that first call before
//    any stream capture on the device.
//  * No cudaMalloc, cudaFree or allocating library routine is called here or
//    on the path below (kernel launches, cudaMemsetAsync and attribute
//    queries only).
#include <stdio.h>

#include <mutex>
#include <string>

#include "../../include/flashgmm.h"
#include "fgmm_internal.cuh"

namespace {

constexpr size_t kScratchBytes = FGMM_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The scratch itself.  A separate translation unit keeps it in its own
// module, so a process that never calls this entry point never loads it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch on the current device; set up once per
// device.  cudaDeviceReset unloads the module that holds the array, so the
// cached address is only valid until the process resets that device; a
// caller that resets a device must not call this entry point afterwards.  Returns FGMM_OK or an FGMM_ERR_* code with the message recorded.
int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fgmm::entry_fail(FGMM_ERR_CUDA, std::string("fgmm_estep_iso_noalloc: cudaGetDevice: ") +
                                               cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fgmm::entry_fail(FGMM_ERR_DEVICE, "fgmm_estep_iso_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fgmm::entry_fail(
          FGMM_ERR_CUDA, std::string("fgmm_estep_iso_noalloc: cudaGetSymbolAddress of the scratch: ") +
                             cudaGetErrorString(e));
    if (reinterpret_cast<uintptr_t>(p) & 255)
      return fgmm::entry_fail(FGMM_ERR_WORKSPACE,
                              "fgmm_estep_iso_noalloc: scratch is not 256-byte aligned");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FGMM_OK;
}

}  // namespace

extern "C" {

int fgmm_estep_iso_noalloc(const float* X, int64_t x_stride_n, int64_t x_stride_d,
                           const float* mu, int64_t mu_stride_k, int64_t mu_stride_d,
                           const float* log_sigma_sq, const float* log_pi, int64_t N, int32_t K,
                           int32_t D, float* logZ, float* Nk, float* mu_acc, float* sig_acc,
                           unsigned flags, void* stream) {
  fgmm::EstepArgs a{X,      x_stride_n, x_stride_d, mu,     mu_stride_k, mu_stride_d,
                    log_sigma_sq, log_pi, N,     K,      D,           logZ,
                    Nk,     mu_acc,     sig_acc,    nullptr, 0,          flags,
                    reinterpret_cast<cudaStream_t>(stream)};
  if (N < 0 || K < 1 || D < 1 || D > fgmm::kGeneralMaxD)
    return fgmm::entry_run_estep(fgmm::kIso, a);  // reports the shape error
  // The device check comes before the shape query, so a device that is not
  // sm_100 reports FGMM_ERR_DEVICE whatever the shape.
  std::string why;
  const int dc = fgmm::entry_check_device(&why);
  if (dc != FGMM_OK) return fgmm::entry_fail(dc, "fgmm_estep_iso_noalloc: " + why);
  // Scratch the path this call takes needs, exactly as fgmm_estep_iso sizes it.
  const bool fast = !(flags & FGMM_FLAG_FORCE_GENERAL) && fgmm::tc_supported(fgmm::kIso, a, nullptr);
  const size_t need = N == 0 ? 0
                      : fast ? fgmm::tc_workspace_bytes(fgmm::kIso, N, K, D)
                             : fgmm::general_workspace_bytes(fgmm::kIso, N, K, D);
  if (need > kScratchBytes) {
    char buf[256];
    snprintf(buf, sizeof buf,
             "fgmm_estep_iso_noalloc: N=%lld K=%d D=%d needs %zu bytes of scratch, more than the "
             "fixed %zu; call fgmm_estep_iso with a workspace instead",
             (long long)N, K, D, need, kScratchBytes);
    return fgmm::entry_fail(FGMM_ERR_WORKSPACE, buf);
  }
  void* scratch = nullptr;
  const int sc = scratch_for_current_device(&scratch);
  if (sc != FGMM_OK) return sc;
  a.ws = scratch;
  a.ws_bytes = kScratchBytes;
  return fgmm::entry_run_estep(fgmm::kIso, a);
}

}  // extern "C"
