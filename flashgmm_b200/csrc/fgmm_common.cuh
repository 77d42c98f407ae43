// Shared helpers for the flashgmm_b200 CUDA library (host + device).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>
#include <atomic>
#include <string>

#include "../../include/flashgmm_b200.h"
#include "fgmm_tcops.cuh"

namespace fgmm {

constexpr double kLog2Pi = 1.8378770664093453;

// Per-host-thread error message behind fgmm_last_error().
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int cuda_fail(cudaError_t e, const char *what);

#define FGMM_CUDA_TRY(expr)                                   \
  do {                                                        \
    cudaError_t _e = (expr);                                  \
    if (_e != cudaSuccess) return ::fgmm::cuda_fail(_e, #expr); \
  } while (0)

// Programmatic dependent launch: the kernel may be scheduled while its predecessor on the
// stream is still finishing (its launch and set-up overlap the predecessor's tail).  Every
// kernel launched this way calls griddep_wait() before it touches global memory that
// earlier work on the stream reads or writes, and griddep_launch() once all its blocks
// have been scheduled, so the next kernel can start setting up.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
#ifdef FGMM_NO_PDL
  cfg.numAttrs = 0;
#else
  cfg.numAttrs = 1;
#endif
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

#define FGMM_LAUNCH_CHECK(what)                               \
  do {                                                        \
    cudaError_t _e = cudaGetLastError();                      \
    if (_e != cudaSuccess) return ::fgmm::cuda_fail(_e, what); \
  } while (0)

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Bump allocator over a caller-provided workspace.
struct Carve {
  char *base;
  size_t off = 0;
  explicit Carve(void *p) : base(static_cast<char *>(p)) {}
  template <class T> T *take(size_t count) {
    off = align_up(off, 256);
    T *p = base ? reinterpret_cast<T *>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
  size_t bytes() const { return align_up(off, 256); }
};

int num_sms();
// Per-device "done" flag for one-time kernel attribute settings (cudaFuncSetAttribute
// applies to the current device only): flag `slot` (< 16) of the current device.
std::atomic<bool> &device_once_flag(int slot);

// Optional per-launch event recording (active only inside fgmm_em_stats_profiled).
struct PhaseTimer {
  static constexpr int kMax = 128;
  cudaEvent_t ev[kMax + 1];
  const char *name[kMax];
  int n = 0;
};
PhaseTimer *&phase_timer();
// Record the end of the launch just issued on `st` (no-op when not profiling).
inline void mark(cudaStream_t st, const char *name) {
  PhaseTimer *t = phase_timer();
  if (t && t->n < PhaseTimer::kMax) {
    t->name[t->n] = name;
    cudaEventRecord(t->ev[++t->n], st);
  }
}
int simt_launches();
int tc_launches(int64_t N, int d, int K);

// Where the M-step is applied in the same launch as the statistics reduction.
struct UpdateOut {
  double n_total;
  float *mu, *var, *log_pi;
  bool floors;
  // Optional (tensor-core family, d <= 128): also write the next iteration's
  // parameter operands for the updated parameters, as tc_prep_params_kernel would
  // (tc.kbp = 0: off).
  TcParamOps tc;
};

// ---- SIMT family (fgmm_simt.cu) ----
size_t simt_workspace_bytes(int64_t N, int d, int K);
int simt_em_stats(const float *X, int64_t N, int d, const float *mu, const float *var,
                  const float *log_pi, int K, double *stats, float *log_norm,
                  void *ws, cudaStream_t stream, const UpdateOut *update = nullptr);

// ---- low-K family (fgmm_lowk.cu): K <= 16, d <= 128, two launches per iteration ----
bool lowk_supported(int64_t N, int d, int K);
int lowk_launches();
size_t lowk_workspace_bytes(int64_t N, int d, int K);
int lowk_em_stats(const float *X, int64_t N, int d, const float *mu, const float *var,
                  const float *log_pi, int K, double *stats, float *log_norm, void *ws,
                  cudaStream_t stream, const UpdateOut *update = nullptr);

// ---- tcgen05 family (fgmm_tc.cu) ----
bool tc_supported(int64_t N, int d, int K);
size_t tc_points_bytes(int64_t N, int d);
size_t tc_workspace_bytes(int64_t N, int d, int K);
int tc_prepare_points(const float *X, int64_t N, int d, void *points, cudaStream_t stream);
// Code of the first bounded-wait failure recorded by a tensor-core kernel (0 = none).
int tc_device_error(bool reset);
int tc_em_stats(const float *X, const void *points, int64_t N, int d, const float *mu,
                const float *var, const float *log_pi, int K, double *stats,
                float *log_norm, void *ws, cudaStream_t stream, const UpdateOut *update = nullptr,
                bool prepared = false);

// ---- shared epilogue kernels (fgmm_update.cu) ----
// Sums per-block fp32 partials [K][slots][W] (rows [s (ds) | sq (ds) | n ...]) and
// per-block log-normalizer sums into the packed fp64 stats vector (one launch); with
// `update`, also writes the updated parameters.
int reduce_partials(const float *partials, int slots, int K, int d, int ds, int W,
                    const double *ln_partials, int ln_slots, double *stats,
                    cudaStream_t stream, const UpdateOut *update = nullptr);
// M-step (floored) that also writes the tensor-core operands of the new values.
int em_update_prep(const double *stats, double n_total, int K, int Kp, int d, float *new_mu,
                   float *new_var, float *new_log_pi, const TcParamOps &op, cudaStream_t stream);
// The sharded fit's update step: em_update_prep into the statistics workspace of
// tc_em_stats for (N, d, K) and these prepared points.
int tc_update_prepare(const double *stats, double n_total, const void *points, int64_t N, int d,
                      int K, float *new_mu, float *new_var, float *new_log_pi, void *ws,
                      cudaStream_t stream);
int em_update(const double *stats, double n_total, int K, int d, float *new_mu,
              float *new_var, float *new_log_pi, cudaStream_t stream, bool floors = true);

// Direct-form parameters: sc = var^-1/2, ms = mu var^-1/2 ([K][d]) and
// lc = log_pi - 1/2 (d log 2pi + sum log var) ([K]) (fgmm_simt.cu).
int prep_direct_params(const float *mu, const float *var, const float *log_pi, int K, int d,
                       float *sc, float *ms, float *lc, cudaStream_t stream);

// ---- E-step / M-step with materialised responsibilities (fgmm_estep.cu, fgmm_simt.cu) ----
size_t estep_workspace_bytes(int64_t N, int d, int K);
int estep(const float *X, int64_t N, int d, const float *mu, const float *var,
          const float *log_pi, int K, float *gamma, float *log_norm, void *ws,
          cudaStream_t stream);
size_t mstep_workspace_bytes(int64_t N, int d, int K);
// Packed fp64 statistics [n | s | sq | 0] of given responsibilities gamma[N][K].
int mstep_stats(const float *X, int64_t N, int d, const float *gamma, int K, double *stats,
                void *ws, cudaStream_t stream);

}  // namespace fgmm
