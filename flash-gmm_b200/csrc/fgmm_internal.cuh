// Internal declarations shared by the libflashgmm_sm100 translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace fgmm {

constexpr double kLog2Pi = 1.8378770664093453;  // log(2 pi)
constexpr double kLog2E = 1.4426950408889634;   // 1 / ln 2

enum Variant { kIso = 0, kDiag = 1, kFull = 2 };

// Element type of X: fp32, or bfloat16 stored as its 16 bits (uint16_t).
enum XType { kXF32 = 0, kXBF16 = 1 };

// X loads widened to fp32 (a bfloat16 is the top half of an fp32: exact).
__device__ __forceinline__ float ldx(const float* p) { return __ldg(p); }
__device__ __forceinline__ float ldx(const uint16_t* p) {
  return __uint_as_float((uint32_t)__ldg(p) << 16);
}
// Four consecutive elements from a 16-byte (fp32) or 8-byte (bf16) aligned address.
__device__ __forceinline__ float4 ldx4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ float4 ldx4(const uint16_t* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}
// Calls f with a null pointer of X's element type (a type tag).
template <class F>
decltype(auto) with_xtype(int xtype, F&& f) {
  if (xtype == kXBF16) return f(static_cast<const uint16_t*>(nullptr));
  return f(static_cast<const float*>(nullptr));
}

// Arguments of one E-step call, as received through the C ABI.
struct EstepArgs {
  const void* X;     // xtype elements
  int64_t sxn, sxd;
  const float* mu;
  int64_t smk, smd;
  const float* cov;  // iso: log_sigma_sq (K); diag: log_sigma_sq (K,D);
                     // full: prec_chol (K,D,D)
  const float* lpi;
  int64_t N;
  int K, D;
  float* logZ;
  float* Nk;
  float* mu_acc;
  float* sig;
  void* ws;
  size_t ws_bytes;
  unsigned flags;
  cudaStream_t stream;
  int xtype = kXF32;
  // X as its element type, and its 16-byte-vector loads allowed (unit
  // feature stride, aligned base, rows of a multiple of 4 elements)
  template <class TX>
  const TX* x() const { return static_cast<const TX*>(X); }
  int x_vec_ok() const {
    const uintptr_t align = xtype == kXBF16 ? 7 : 15;
    return sxd == 1 && (reinterpret_cast<uintptr_t>(X) & align) == 0 && sxn % 4 == 0;
  }
};

// Bump allocator over the caller's workspace; every block 256-byte aligned.
struct WsCarve {
  char* base;
  size_t used = 0;
  explicit WsCarve(void* p) : base(static_cast<char*>(p)) {}
  template <typename T>
  T* take(size_t count) {
    size_t off = (used + 255) & ~size_t(255);
    used = off + count * sizeof(T);
    return base ? reinterpret_cast<T*>(base + off) : nullptr;
  }
};

// General (CUDA-core) kernels: any strides, any K, D <= kGeneralMaxD.
constexpr int kGeneralMaxD = 256;
constexpr int kGeneralMaxDFull = 128;
size_t general_workspace_bytes(int variant, int64_t N, int K, int D);
cudaError_t general_estep(int variant, const EstepArgs& a);

// Tensor-core (tcgen05) isotropic / diagonal path.
bool tc_supported(int variant, const EstepArgs& a, std::string* why);
size_t tc_workspace_bytes(int variant, int64_t N, int K, int D);
cudaError_t tc_estep(int variant, const EstepArgs& a);

// Tensor-core full-covariance path (fgmm_tc_full.cu).
bool full_tc_supported(const EstepArgs& a);
size_t full_tc_workspace_bytes(int64_t N, int K, int D);
cudaError_t full_tc_estep(const EstepArgs& a);

// c_d = mean_k mu_kd (0 for d >= D) and *amax |= the largest |mu_kd - c_d|
// and |x_nd - c_d| over an evenly spaced sample of kScaleSample rows (float
// bits, atomicMax; *amax must start at 0): the X scale of the split passes.
// One launch of Dp blocks on `stream`.
constexpr int64_t kScaleSample = 4096;
void launch_centre(const EstepArgs& a, int Dp, float* cvec, int* amax, cudaStream_t stream);

// Row generator for the streaming configuration.
cudaError_t generate_iso_rows(float* X, const int64_t* row_ids, int64_t row0,
                              int64_t nrows, int D, const float* centres, int K,
                              uint64_t seed, cudaStream_t stream);

int num_sms();

// Raise (never lower) the dynamic shared-memory limit of `kernel` on the
// current device to at least `bytes`; thread-safe.
cudaError_t ensure_dynamic_smem(const void* kernel, size_t bytes);

// Shared by the extern "C" entry points: record a failure message for
// fgmm_last_error(), the sm_100 device check, and the validated E-step
// dispatch (argument checks, workspace check, tensor-core or general path).
int entry_fail(int code, const std::string& msg);
int entry_check_device(std::string* why);
int entry_run_estep(int variant, const EstepArgs& a);

// Launch accounting and the optional profiling events around the dominant
// kernel (see fgmm_launch_count / fgmm_set_profile_events).
void count_launches(int n);
void profile_mark(bool stop, cudaStream_t stream);

}  // namespace fgmm
