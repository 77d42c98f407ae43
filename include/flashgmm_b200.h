/*
 * flashgmm_b200.h -- C ABI of the B200 (sm_100a) fused diagonal-covariance EM
 * iteration.  Plain pointers and sizes only; every pointer argument named
 * X / mu / var / log_pi / new_* / stats / log_normalizer / gamma / workspace /
 * points is DEVICE memory on the current CUDA device, and `stream` is a
 * cudaStream_t (NULL = legacy default stream).  All calls are asynchronous with
 * respect to the host unless stated otherwise.
 *
 * Layouts: X[N][d], mu[K][d], var[K][d], gamma[N][K] are row-major fp32;
 * log_pi[K], log_normalizer[N] fp32.  `stats` is the packed fp64 sufficient
 * statistics vector of length fgmm_stats_len(K, d):
 *     [ n_k (K) | s_k (K*d) | sq_k (K*d) | sum_n log_normalizer_n (1) ]
 * which is what a multi-GPU caller sums across ranks between fgmm_em_stats and
 * fgmm_em_update.
 *
 * Return value: FGMM_OK (0) or an FGMM_ERR_* code; fgmm_last_error() gives the
 * message of the last failure on the calling host thread.
 */
#ifndef FLASHGMM_B200_H_
#define FLASHGMM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FGMM_OK 0
#define FGMM_ERR_INVALID 1      /* bad shape / null pointer / misaligned pointer */
#define FGMM_ERR_UNSUPPORTED 2  /* shape outside what the kernels handle (d > 256) */
#define FGMM_ERR_WORKSPACE 3    /* workspace smaller than the *_bytes query */
#define FGMM_ERR_CUDA 4         /* a CUDA runtime call or kernel launch failed */

/* Kernel families fgmm_em_stats can run. */
#define FGMM_FAMILY_AUTO 0      /* low-K kernel for K <= 16, d <= 128, K d <= 512; else tcgen05
                                   where the shape allows (d <= 128); else SIMT */
#define FGMM_FAMILY_SIMT 1      /* force the generic fp32 CUDA-core kernels */
#define FGMM_FAMILY_TC 2        /* require the tcgen05 kernels (error if the shape is outside them) */
#define FGMM_FAMILY_LOWK 3      /* require the fused low-K kernel (K <= 16, d <= 128; error otherwise) */

const char *fgmm_last_error(void);
int fgmm_version(void);

/* Select the kernel family used by subsequent fgmm_em_stats / fgmm_em_fused
 * calls in this process (default FGMM_FAMILY_AUTO).  Returns the previous value. */
int fgmm_set_family(int family);
/* Which family fgmm_em_stats would run for this shape under the current setting
 * (FGMM_FAMILY_SIMT, FGMM_FAMILY_TC or FGMM_FAMILY_LOWK), or -1 if the shape is
 * unsupported. */
int fgmm_family_for(int64_t N, int32_t d, int32_t K);

/* Length (in doubles) of the packed statistics vector: K*(2d+1)+1. */
int64_t fgmm_stats_len(int32_t K, int32_t d);

/* Bytes of the "prepared points" buffer for X[N][d]: the per-point tensor-core
 * operand rows [x^2 | x] split into tf32 hi/lo parts.  X is constant over an EM
 * fit, so a caller may prepare once and pass `points` to every fgmm_em_stats.
 * Returns 0 when the shape runs on the SIMT family (no preparation needed). */
size_t fgmm_points_bytes(int64_t N, int32_t d, int32_t K);
int fgmm_prepare_points(const float *X, int64_t N, int32_t d, int32_t K,
                        void *points, size_t points_bytes, void *stream);

/* Scratch needed by fgmm_em_stats (parameter operands, per-block partial
 * statistics and log-sum-exp partials).  256-byte aligned pointer required. */
size_t fgmm_em_stats_workspace_bytes(int64_t N, int32_t d, int32_t K);

/* Pass 1 (online log-sum-exp -> log_normalizer[N]) and Pass 2 (responsibilities
 * recomputed on chip, accumulated into n_k, s_k = gamma^T X, sq_k = gamma^T X^2)
 * over the N local points.  Writes `stats` (fp64, see above) and
 * `log_normalizer`.  `points` may be NULL, in which case the tensor-core family
 * prepares the operands inside `workspace` (which must then be at least
 * fgmm_em_fused_workspace_bytes).
 * Replaces the first three launches of flash_em_fused_cuda
 * (reference flash_gmm/csrc/flash_gmm_cuda.cu:418-493: precompute_params_kernel,
 * flash_log_normalizer_v2_kernel, flash_accumulate_stats_v2_kernel). */
int fgmm_em_stats(const float *X, const void *points, int64_t N, int32_t d,
                  const float *mu, const float *var, const float *log_pi, int32_t K,
                  double *stats, float *log_normalizer,
                  void *workspace, size_t workspace_bytes, void *stream);

/* M-step from (globally summed) statistics: mu = s/max(n,1e-8),
 * var = max(sq/n - mu^2, 1e-6), log_pi = log(max(n/n_total, 1e-8)).
 * Replaces update_params_kernel (reference flash_gmm/csrc/flash_gmm_cuda.cu:298-322,
 * launched at :496-501) with the same floors as flash_gmm/csrc/flash_gmm_cpu.cpp:270-284. */
int fgmm_em_update(const double *stats, double n_total, int32_t K, int32_t d,
                   float *new_mu, float *new_var, float *new_log_pi, void *stream);

/* fgmm_em_update with options.  flags = 0 is fgmm_em_update.  FGMM_UPDATE_NO_FLOORS
 * applies the pure-Python model's update instead (reference flash_gmm/flash_gmm.py:162-169,
 * FlashGMM._fused_em_step): mu = s/n, var = max(sq/n - mu^2, 1e-6), log_pi = log(n/n_total),
 * with no floor on n or on the weight (an empty component gives NaN / -inf, as there). */
#define FGMM_UPDATE_NO_FLOORS 1
int fgmm_em_update_ex(const double *stats, double n_total, int32_t K, int32_t d, int32_t flags,
                      float *new_mu, float *new_var, float *new_log_pi, void *stream);

/* One EM iteration on one device over prepared points: fgmm_em_stats followed by
 * the M-step of fgmm_em_update (n_total = N), the update applied inside the
 * statistics reduction's launch.  `stats` and `log_normalizer` are written as by
 * fgmm_em_stats (the log-likelihood is stats[K(2d+1)] / N); the new parameters may
 * alias mu / var / log_pi.  The same launch also leaves in `workspace` the
 * tensor-core operands of the new parameters: a following call whose mu / var /
 * log_pi are exactly this call's outputs (unchanged in between) and whose workspace
 * is the same may pass FGMM_STEP_PREPARED in `flags` to skip preparing them again
 * (tensor-core family with prepared points only; otherwise FGMM_ERR_INVALID).
 * Replaces one pass of the reference's fit loop (flash_gmm/native_wrapper.py:128-146
 * calling flash_em_fused on the same X every iteration), without re-preparing the
 * point operands. */
#define FGMM_STEP_PREPARED 1
int fgmm_em_step(const float *X, const void *points, int64_t N, int32_t d,
                 const float *mu, const float *var, const float *log_pi, int32_t K,
                 float *new_mu, float *new_var, float *new_log_pi,
                 double *stats, float *log_normalizer,
                 void *workspace, size_t workspace_bytes, int32_t flags, void *stream);

/* fgmm_em_stats with flags: FGMM_STEP_PREPARED reuses the parameter operands that
 * fgmm_em_update_prepared left in `workspace` for exactly these mu / var / log_pi
 * (tensor-core family with prepared points; otherwise FGMM_ERR_INVALID).  The per-rank
 * statistics pass of a sharded fit; like fgmm_em_stats it replaces
 * flash_gmm/csrc/flash_gmm_cuda.cu:418-493. */
int fgmm_em_stats_ex(const float *X, const void *points, int64_t N, int32_t d,
                     const float *mu, const float *var, const float *log_pi, int32_t K,
                     double *stats, float *log_normalizer,
                     void *workspace, size_t workspace_bytes, int32_t flags, void *stream);

/* The update step of a sharded fit, after the statistics all-reduce: fgmm_em_update's
 * M-step (floors as there, flash_gmm/csrc/flash_gmm_cuda.cu:298-322) in one launch that
 * also writes the tensor-core operands of the new parameters into `workspace` (the
 * fgmm_em_stats workspace of this rank's N local points), so the next
 * fgmm_em_stats_ex(..., FGMM_STEP_PREPARED) skips preparing them.  Tensor-core family
 * only. */
int fgmm_em_update_prepared(const double *stats, double n_total, const void *points, int64_t N,
                            int32_t d, int32_t K, float *new_mu, float *new_var,
                            float *new_log_pi, void *workspace, size_t workspace_bytes,
                            void *stream);

/* One fused EM iteration on one device: stats + update.  The drop-in for the
 * reference's op `flash_em_fused(X, mu, var, log_pi, BN, BK)`
 * (flash_gmm/csrc/binding.cpp:62-76 dispatching to flash_em_fused_cuda,
 * flash_gmm/csrc/flash_gmm_cuda.cu:402-504).  The reference's BN/BK tile hints
 * have no counterpart: tile shapes are fixed by the kernels. */
size_t fgmm_em_fused_workspace_bytes(int64_t N, int32_t d, int32_t K);
int fgmm_em_fused(const float *X, int64_t N, int32_t d,
                  const float *mu, const float *var, const float *log_pi, int32_t K,
                  float *new_mu, float *new_var, float *new_log_pi, float *log_normalizer,
                  void *workspace, size_t workspace_bytes, void *stream);

/* E-step with materialised responsibilities: gamma[N][K] (row-major) and
 * log_normalizer[N], the log-likelihood in the reference's direct form.  The
 * drop-in for the ops `standard_e_step(X, mu, var, log_pi)` and
 * `flash_e_step(X, mu, var, log_pi, BK)` (flash_gmm/csrc/binding.cpp:35-60;
 * CUDA standard_e_step_cuda, flash_gmm/csrc/flash_gmm_cuda.cu:328-400; the
 * reference runs flash_e_step on the CPU only, flash_gmm_cpu.cpp:108-168). */
size_t fgmm_e_step_workspace_bytes(int64_t N, int32_t d, int32_t K);
int fgmm_e_step(const float *X, int64_t N, int32_t d,
                const float *mu, const float *var, const float *log_pi, int32_t K,
                float *gamma, float *log_normalizer,
                void *workspace, size_t workspace_bytes, void *stream);

/* M-step from given responsibilities gamma[N][K]: the drop-in for the op
 * `standard_m_step(X, gamma)` (flash_gmm/csrc/binding.cpp:78-92; CPU
 * flash_gmm_cpu.cpp:292-311): mu = gamma^T X / n_k, var = max(gamma^T X^2 / n_k
 * - mu^2, 1e-6), log_pi = log(n_k / N), n_k = sum_n gamma[n][k], with no floor on
 * n_k (as in the reference).  Statistics are summed in fp64. */
size_t fgmm_m_step_workspace_bytes(int64_t N, int32_t d, int32_t K);
int fgmm_m_step(const float *X, int64_t N, int32_t d, const float *gamma, int32_t K,
                float *new_mu, float *new_var, float *new_log_pi,
                void *workspace, size_t workspace_bytes, void *stream);

/* Synchronises the device and returns the code of the first failure a
 * tensor-core kernel recorded (0 = none): every wait inside those kernels is
 * bounded, and a wait that runs out records its code here and makes the kernel
 * return instead of hanging.  reset != 0 clears the code.  Negative on a CUDA
 * error.  Has no counterpart in the reference (its kernels have no waits). */
int fgmm_device_error(int reset);

/* Number of kernel launches one fgmm_em_stats call makes for this shape
 * (fgmm_em_update adds one more). */
int fgmm_em_stats_launches(int64_t N, int32_t d, int32_t K);

/* Profiling variant of fgmm_em_stats: identical launches, with a CUDA event
 * recorded on `stream` before the first and after every launch.  Synchronises
 * the stream, then writes the duration (ms) of each launch into
 * launch_ms[0 .. min(n, launches, 128)-1] and, if names != NULL, a static name
 * string per launch.  Returns the status of the wrapped call.  Has no
 * counterpart in the reference (its launcher exposes no timing). */
int fgmm_em_stats_profiled(const float *X, const void *points, int64_t N, int32_t d,
                           const float *mu, const float *var, const float *log_pi, int32_t K,
                           double *stats, float *log_normalizer,
                           void *workspace, size_t workspace_bytes, void *stream,
                           float *launch_ms, const char **names, int32_t n);

/* Size of the fixed device scratch array behind fgmm_em_fused_static. */
#define FGMM_STATIC_SCRATCH_BYTES (16u << 20)

/* One fused EM iteration (same outputs as fgmm_em_fused, computed by the generic
 * fp32 CUDA-core kernels) that allocates no device memory, for callers that cannot
 * call cudaMalloc: code running inside another framework's memory pool, or a process
 * whose device footprint must stay fixed after start-up.  Its scratch is a fixed
 * FGMM_STATIC_SCRATCH_BYTES (16 MiB) device array that every GPU loading this library
 * holds until the process exits; shapes needing more are rejected with
 * FGMM_ERR_WORKSPACE.  The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress), so make that first call before any stream capture.
 * All calls share the array and it keeps the last call's contents: calls that overlap
 * on the GPU race.  No counterpart in the reference (whose launcher allocates its
 * scratch with torch on every call). */
int fgmm_em_fused_static(const float *X, int64_t N, int32_t d,
                         const float *mu, const float *var, const float *log_pi, int32_t K,
                         float *new_mu, float *new_var, float *new_log_pi, float *log_normalizer,
                         void *stream);

#ifdef __cplusplus
}
#endif
#endif /* FLASHGMM_B200_H_ */
