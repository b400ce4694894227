/*
 * flashgmm.h -- C ABI of the B200 (sm_100a) Gaussian-mixture E-step library
 * libflashgmm_sm100.so.
 *
 * One entry point per covariance family.  Each replaces, as one call, the
 * host wrapper + two Triton launches of the reference:
 *
 *   fgmm_estep_iso   <- flash_gmm.py:173-217        (flash_gmm_estep, fp32)
 *                       flash_gmm_h100.py:254-328   (flash_gmm_estep, H100)
 *   fgmm_estep_diag  <- flash_gmm_diag_h100.py:305-384 (flash_gmm_estep_diag)
 *   fgmm_estep_full  <- flash_gmm_full_h100.py:235-336 (flash_gmm_estep_full)
 *
 * Conventions (all entry points):
 *  - Every array argument is a DEVICE pointer owned by the caller.  float32.
 *  - X is (N, D) with element strides (x_stride_n, x_stride_d), as the
 *    reference passes X.stride() through (flash_gmm.py:202).  mu is (K, D)
 *    with strides (mu_stride_k, mu_stride_d).  All other inputs are
 *    contiguous: log_sigma_sq (K) iso / (K, D) diag, prec_chol (K, D, D),
 *    log_pi (K).
 *  - Outputs are contiguous and fully written by the call (no pre-zeroing):
 *      logZ (N)       natural-log per-sample normaliser
 *      Nk (K)         sum_n r_nk
 *      mu_acc (K, D)  sum_n r_nk x_n
 *      sig            iso : (K)      sum_n r_nk ||x_n - mu_k||^2
 *                     diag: (K, D)   sum_n r_nk (x_nd - mu_kd)^2
 *                     full: (K,D,D)  sum_n r_nk x_n x_n^T (uncentred)
 *    With FGMM_FLAG_ACCUMULATE the Nk/mu_acc/sig results are ADDED to the
 *    values already in those buffers (logZ is still overwritten); this is the
 *    chunk-summing step of the reference's streaming recipe (README.md:81-103).
 *  - workspace: device scratch of at least fgmm_workspace_bytes(...) bytes,
 *    256-byte aligned.  It holds per-CTA partial statistics, which a second
 *    kernel reduces in a fixed order: results are bitwise reproducible
 *    run-to-run (the reference's tl.atomic_add accumulation is not).
 *  - stream: a cudaStream_t passed as void*; NULL = legacy default stream.
 *    The call is asynchronous on that stream and never synchronises.  Large
 *    isotropic / diagonal calls (>= 2048 row tiles) fork two library-owned
 *    streams (one pair per host thread and device, created on first use) and
 *    join back to `stream` with events: work the caller enqueues on `stream`
 *    after the call sees all of its results.
 *  - Return value: FGMM_OK (0) or one of the FGMM_ERR_* codes; no C++
 *    exception crosses the ABI.  fgmm_last_error() gives a message for the
 *    last failing call on the calling thread.
 *  - Device-side failures cannot change the return value (the call has
 *    returned before its kernels run).  The tensor-core kernels check on the
 *    device that (a) every scaled value of X is finite and fits fp16's range -- X is scaled
 *    by one power of two chosen from the means and an evenly spaced sample
 *    of 4096 rows, which leaves room for rows about 2,000x (isotropic, full)
 *    or 30x (diagonal, whose features include squares) farther from the
 *    means' centre than any of those -- and (b) that every bounded wait
 *    completed.  If either fails, logZ may be wrong and Nk, mu_acc and sig
 *    are all NaN.  The first int32 of the workspace is the call's status
 *    word: once the call's work on `stream` has completed it reads 0, or
 *    FGMM_STATUS_RANGE for (a), or another nonzero value for (b).  The
 *    no-workspace entry fgmm_estep_iso_noalloc signals them through the NaN
 *    outputs only.
 */
#ifndef FLASHGMM_H_
#define FLASHGMM_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FGMM_API __attribute__((visibility("default")))
#else
#define FGMM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FGMM_OK 0
#define FGMM_ERR_ARG 1          /* bad shape, stride or null pointer      */
#define FGMM_ERR_WORKSPACE 2    /* workspace missing, small or unaligned   */
#define FGMM_ERR_UNSUPPORTED 3  /* shape outside what any kernel handles   */
#define FGMM_ERR_CUDA 4         /* CUDA launch / runtime error             */
#define FGMM_ERR_DEVICE 5       /* device is not sm_100                    */

/* Bit of the workspace status word: a scaled value of X left fp16's range. */
#define FGMM_STATUS_RANGE 0x10000

#define FGMM_VARIANT_ISO 0
#define FGMM_VARIANT_DIAG 1
#define FGMM_VARIANT_FULL 2

#define FGMM_FLAG_ACCUMULATE 1u /* add Nk/mu_acc/sig into the outputs      */

#define FGMM_X_F32 0            /* X element types of fgmm_estep_x */
#define FGMM_X_BF16 1
#define FGMM_FLAG_FORCE_GENERAL 2u /* use the general (non-tensor-core)
                                      kernels even when the fast path applies */

/* Library version, major*10000 + minor*100 + patch. */
FGMM_API int fgmm_version(void);

/* Message describing the last failed call on this thread ("" if none). */
FGMM_API const char* fgmm_last_error(void);

/* Bytes of device workspace the entry point for `variant` needs at this
 * shape (0 is a valid answer).  Replaces the reference's internal torch
 * allocations of padded copies and accumulators (e.g. flash_gmm_h100.py:
 * 277-298).  Pure host function: touches no device state. */
FGMM_API size_t fgmm_workspace_bytes(int variant, int64_t N, int32_t K, int32_t D);

/* Isotropic E-step.  Replaces flash_gmm.py:173-217 and
 * flash_gmm_h100.py:254-328. */
FGMM_API int fgmm_estep_iso(const float* X, int64_t x_stride_n, int64_t x_stride_d,
                   const float* mu, int64_t mu_stride_k, int64_t mu_stride_d,
                   const float* log_sigma_sq, const float* log_pi,
                   int64_t N, int32_t K, int32_t D,
                   float* logZ, float* Nk, float* mu_acc, float* sig_acc,
                   void* workspace, size_t workspace_bytes,
                   unsigned flags, void* stream);

/* Diagonal-covariance E-step; log_sigma_sq is (K, D).  Replaces
 * flash_gmm_diag_h100.py:305-384 (without its pass-2 slab overlap). */
FGMM_API int fgmm_estep_diag(const float* X, int64_t x_stride_n, int64_t x_stride_d,
                    const float* mu, int64_t mu_stride_k, int64_t mu_stride_d,
                    const float* log_sigma_sq, const float* log_pi,
                    int64_t N, int32_t K, int32_t D,
                    float* logZ, float* Nk, float* mu_acc, float* sig_acc,
                    void* workspace, size_t workspace_bytes,
                    unsigned flags, void* stream);

/* Full-covariance E-step; prec_chol is (K, D, D) with
 * prec_chol[k] @ prec_chol[k]^T = Sigma_k^-1.  Replaces
 * flash_gmm_full_h100.py:235-336. */
FGMM_API int fgmm_estep_full(const float* X, int64_t x_stride_n, int64_t x_stride_d,
                    const float* mu, int64_t mu_stride_k, int64_t mu_stride_d,
                    const float* prec_chol, const float* log_pi,
                    int64_t N, int32_t K, int32_t D,
                    float* logZ, float* Nk, float* mu_acc, float* sig_outer,
                    void* workspace, size_t workspace_bytes,
                    unsigned flags, void* stream);

/* Any variant (FGMM_VARIANT_*) with X stored as x_type elements: FGMM_X_F32
 * (the three entries above) or FGMM_X_BF16 (bfloat16 bit patterns, 2 bytes
 * each; strides in elements).  A bfloat16 X is widened exactly to fp32 as it
 * is read, so the results equal those of the fp32 entries on the widened
 * values.  No counterpart in the reference: its H100 module casts X to
 * bfloat16 on the host side of each call (flash_gmm_h100.py:272-276); here a
 * caller that already holds bfloat16 data passes it as is.  cov is
 * log_sigma_sq (iso, diag) or prec_chol (full); sig is sig_acc or
 * sig_outer. */
FGMM_API int fgmm_estep_x(int variant, int x_type, const void* X, int64_t x_stride_n,
                 int64_t x_stride_d, const float* mu, int64_t mu_stride_k,
                 int64_t mu_stride_d, const float* cov, const float* log_pi,
                 int64_t N, int32_t K, int32_t D,
                 float* logZ, float* Nk, float* mu_acc, float* sig,
                 void* workspace, size_t workspace_bytes,
                 unsigned flags, void* stream);

/* Isotropic E-step that allocates nothing and takes no workspace: same
 * arguments, results and paths as fgmm_estep_iso, with the scratch in a
 * fixed device array of FGMM_NOALLOC_SCRATCH_BYTES per device owned by the
 * library.  For callers that cannot allocate device memory at the call site
 * (a host runtime whose device memory belongs to another pool, or a loop
 * that must not call cudaMalloc).  No counterpart in the reference.
 *  - Shapes whose workspace exceeds the scratch return FGMM_ERR_WORKSPACE
 *    (about 100,000 rows at D = 128 on the tensor-core path; the general
 *    kernels' scratch does not grow with N).
 *  - Nothing has to be zeroed beforehand.
 *  - The first call on a device does a one-time set-up (looks up the
 *    array's device address); make it before any stream capture.
 *  - All calls on one device share the array: calls that may overlap in
 *    time (different streams or unordered host threads) race. */
#define FGMM_NOALLOC_SCRATCH_BYTES (64u << 20)
FGMM_API int fgmm_estep_iso_noalloc(const float* X, int64_t x_stride_n, int64_t x_stride_d,
                   const float* mu, int64_t mu_stride_k, int64_t mu_stride_d,
                   const float* log_sigma_sq, const float* log_pi,
                   int64_t N, int32_t K, int32_t D,
                   float* logZ, float* Nk, float* mu_acc, float* sig_acc,
                   unsigned flags, void* stream);

/* Number of kernels this library has launched in this process (all devices,
 * all threads).  Lets a caller count the launches inside a timed region. */
FGMM_API uint64_t fgmm_launch_count(void);

/* Register two cudaEvent_t (passed as void*) that subsequent E-step calls on
 * this thread record on their stream immediately before and after the
 * dominant (tensor-core or pass-2) kernel; NULL, NULL disables.  Used by the
 * benchmark to time that kernel alone with CUDA events. */
FGMM_API void fgmm_set_profile_events(void* start_event, void* stop_event);

/* Fill rows of the isotropic mixture used by the streaming configuration:
 * x_n = centres[c(n)] + z_n, z_n ~ N(0, I), with c(n) uniform over K and
 * every value a pure function of (seed, n, d) -- the same global row n gets
 * the same values whatever the sharding.  Output row i is global row
 * row_ids[i] when row_ids (device, int64) is non-NULL, else row0 + i.
 * X is (nrows, D) contiguous; centres is (K, D) contiguous.  This is the
 * on-device stand-in for the reference's host->device chunk loop
 * (README.md:81-103); it has no counterpart kernel in the reference. */
FGMM_API int fgmm_generate_iso_rows(float* X, const int64_t* row_ids, int64_t row0,
                           int64_t nrows, int32_t D, const float* centres,
                           int32_t K, uint64_t seed, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHGMM_H_ */
