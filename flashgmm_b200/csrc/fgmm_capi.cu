// extern "C" entry points declared in include/flashgmm_b200.h.
#include <cstdio>
#include <atomic>
#include <mutex>
#include "fgmm_common.cuh"

namespace fgmm {

static thread_local std::string g_err;
static int g_family = FGMM_FAMILY_AUTO;

void set_error(const std::string &m) { g_err = m; }
int fail(int code, const std::string &m) {
  g_err = m;
  return code;
}
int cuda_fail(cudaError_t e, const char *what) {
  g_err = std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e);
  return FGMM_ERR_CUDA;
}

PhaseTimer *&phase_timer() {
  static thread_local PhaseTimer *t = nullptr;
  return t;
}

// Caches shared by every host thread: atomics, so concurrent first calls on one device
// race benignly (both compute the same value) and never tear.
int num_sms() {
  static std::atomic<int> cached[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int v = cached[dev].load(std::memory_order_acquire);
  if (!v) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    cached[dev].store(v, std::memory_order_release);
  }
  return v;
}

std::atomic<bool> &device_once_flag(int slot) {
  static std::atomic<bool> flags[64][16];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  return flags[dev][slot & 15];
}

static int check_shape(int64_t N, int d, int K) {
  if (N < 1 || K < 1 || d < 1)
    return fail(FGMM_ERR_INVALID, "N, K and d must all be >= 1 (got N=" + std::to_string(N) +
                                      " K=" + std::to_string(K) + " d=" + std::to_string(d) + ")");
  if (d > 256) return fail(FGMM_ERR_UNSUPPORTED, "d > 256 is not supported (got d=" + std::to_string(d) + ")");
  if (N > ((int64_t)1 << 40)) return fail(FGMM_ERR_INVALID, "N too large");
  return FGMM_OK;
}

static bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static int resolve_family(int64_t N, int d, int K) {
  if (N < 1 || K < 1 || d < 1 || d > 256) return -1;
  const bool tc = tc_supported(N, d, K);
  const bool lowk = lowk_supported(N, d, K);
  if (g_family == FGMM_FAMILY_SIMT) return FGMM_FAMILY_SIMT;
  if (g_family == FGMM_FAMILY_TC) return tc ? FGMM_FAMILY_TC : -1;
  if (g_family == FGMM_FAMILY_LOWK) return lowk ? FGMM_FAMILY_LOWK : -1;
  // the fused low-K kernel measured faster than the tensor-core family up to K d = 512
  if (lowk && (int64_t)K * d <= 512) return FGMM_FAMILY_LOWK;
  return tc ? FGMM_FAMILY_TC : FGMM_FAMILY_SIMT;
}

}  // namespace fgmm

using namespace fgmm;

extern "C" {

const char *fgmm_last_error(void) { return g_err.c_str(); }
int fgmm_version(void) { return 10000; }

int fgmm_set_family(int family) {
  int prev = g_family;
  if (family == FGMM_FAMILY_AUTO || family == FGMM_FAMILY_SIMT || family == FGMM_FAMILY_TC ||
      family == FGMM_FAMILY_LOWK)
    g_family = family;
  return prev;
}

int fgmm_family_for(int64_t N, int32_t d, int32_t K) { return resolve_family(N, d, K); }

int64_t fgmm_stats_len(int32_t K, int32_t d) { return (int64_t)K * (2 * (int64_t)d + 1) + 1; }

size_t fgmm_points_bytes(int64_t N, int32_t d, int32_t K) {
  if (resolve_family(N, d, K) != FGMM_FAMILY_TC) return 0;
  return tc_points_bytes(N, d);
}

int fgmm_prepare_points(const float *X, int64_t N, int32_t d, int32_t K, void *points,
                        size_t points_bytes, void *stream) {
  int rc = check_shape(N, d, K);
  if (rc) return rc;
  if (resolve_family(N, d, K) != FGMM_FAMILY_TC) return FGMM_OK;  // nothing to prepare
  if (!X || !points) return fail(FGMM_ERR_INVALID, "null pointer");
  if (!aligned(points, 256)) return fail(FGMM_ERR_INVALID, "points must be 256-byte aligned");
  if (points_bytes < tc_points_bytes(N, d)) return fail(FGMM_ERR_WORKSPACE, "points buffer too small");
  return tc_prepare_points(X, N, d, points, (cudaStream_t)stream);
}

size_t fgmm_em_stats_workspace_bytes(int64_t N, int32_t d, int32_t K) {
  int fam = resolve_family(N, d, K);
  if (fam == FGMM_FAMILY_TC) return tc_workspace_bytes(N, d, K);
  if (fam == FGMM_FAMILY_SIMT) return simt_workspace_bytes(N, d, K);
  if (fam == FGMM_FAMILY_LOWK) return lowk_workspace_bytes(N, d, K);
  return 0;
}

namespace {
// fgmm_em_stats, optionally with the M-step applied in the statistics reduction's launch.
int em_stats_impl(const float *X, const void *points, int64_t N, int32_t d, const float *mu,
                  const float *var, const float *log_pi, int32_t K, double *stats,
                  float *log_normalizer, void *workspace, size_t workspace_bytes, void *stream,
                  const fgmm::UpdateOut *update, bool prepared = false) {
  int rc = check_shape(N, d, K);
  if (rc) return rc;
  if (!X || !mu || !var || !log_pi || !stats || !log_normalizer || !workspace)
    return fail(FGMM_ERR_INVALID, "null pointer argument");
  if (!aligned(workspace, 256)) return fail(FGMM_ERR_INVALID, "workspace must be 256-byte aligned");
  if (!aligned(X, 16)) return fail(FGMM_ERR_INVALID, "X must be 16-byte aligned");
  const int fam = resolve_family(N, d, K);
  if (fam < 0) return fail(FGMM_ERR_UNSUPPORTED, "shape not supported by the requested kernel family");
  cudaStream_t st = (cudaStream_t)stream;
  if (fam == FGMM_FAMILY_SIMT) {
    if (workspace_bytes < simt_workspace_bytes(N, d, K))
      return fail(FGMM_ERR_WORKSPACE, "workspace too small");
    return simt_em_stats(X, N, d, mu, var, log_pi, K, stats, log_normalizer, workspace, st, update);
  }
  if (fam == FGMM_FAMILY_LOWK) {
    if (workspace_bytes < lowk_workspace_bytes(N, d, K))
      return fail(FGMM_ERR_WORKSPACE, "workspace too small");
    return lowk_em_stats(X, N, d, mu, var, log_pi, K, stats, log_normalizer, workspace, st, update);
  }
  size_t need = tc_workspace_bytes(N, d, K);
  const void *pts = points;
  if (!pts) {
    size_t pb = tc_points_bytes(N, d);
    if (workspace_bytes < need + pb)
      return fail(FGMM_ERR_WORKSPACE, "workspace too small to prepare points in place");
    void *p = static_cast<char *>(workspace) + need;
    rc = tc_prepare_points(X, N, d, p, st);
    if (rc) return rc;
    pts = p;
  } else if (workspace_bytes < need) {
    return fail(FGMM_ERR_WORKSPACE, "workspace too small");
  }
  return tc_em_stats(X, pts, N, d, mu, var, log_pi, K, stats, log_normalizer, workspace, st, update,
                     prepared);
}
}  // namespace

int fgmm_em_stats(const float *X, const void *points, int64_t N, int32_t d, const float *mu,
                  const float *var, const float *log_pi, int32_t K, double *stats,
                  float *log_normalizer, void *workspace, size_t workspace_bytes, void *stream) {
  return em_stats_impl(X, points, N, d, mu, var, log_pi, K, stats, log_normalizer, workspace,
                       workspace_bytes, stream, nullptr);
}

int fgmm_em_stats_ex(const float *X, const void *points, int64_t N, int32_t d, const float *mu,
                     const float *var, const float *log_pi, int32_t K, double *stats,
                     float *log_normalizer, void *workspace, size_t workspace_bytes, int32_t flags,
                     void *stream) {
  if (flags & ~FGMM_STEP_PREPARED) return fail(FGMM_ERR_INVALID, "unknown flags");
  const bool prepared = (flags & FGMM_STEP_PREPARED) != 0;
  if (prepared && (!points || resolve_family(N, d, K) != FGMM_FAMILY_TC))
    return fail(FGMM_ERR_INVALID, "FGMM_STEP_PREPARED needs the tensor-core family and prepared points");
  return em_stats_impl(X, points, N, d, mu, var, log_pi, K, stats, log_normalizer, workspace,
                       workspace_bytes, stream, nullptr, prepared);
}

int fgmm_em_update_prepared(const double *stats, double n_total, const void *points, int64_t N,
                            int32_t d, int32_t K, float *new_mu, float *new_var, float *new_log_pi,
                            void *workspace, size_t workspace_bytes, void *stream) {
  int rc = check_shape(N, d, K);
  if (rc) return rc;
  if (!stats || !points || !new_mu || !new_var || !new_log_pi || !workspace)
    return fail(FGMM_ERR_INVALID, "null pointer argument");
  if (!(n_total > 0)) return fail(FGMM_ERR_INVALID, "n_total must be > 0");
  if (resolve_family(N, d, K) != FGMM_FAMILY_TC)
    return fail(FGMM_ERR_INVALID, "fgmm_em_update_prepared needs the tensor-core family");
  if (workspace_bytes < tc_workspace_bytes(N, d, K)) return fail(FGMM_ERR_WORKSPACE, "workspace too small");
  return tc_update_prepare(stats, n_total, points, N, d, K, new_mu, new_var, new_log_pi, workspace,
                           (cudaStream_t)stream);
}

int fgmm_em_step(const float *X, const void *points, int64_t N, int32_t d, const float *mu,
                 const float *var, const float *log_pi, int32_t K, float *new_mu, float *new_var,
                 float *new_log_pi, double *stats, float *log_normalizer, void *workspace,
                 size_t workspace_bytes, int32_t flags, void *stream) {
  if (!new_mu || !new_var || !new_log_pi) return fail(FGMM_ERR_INVALID, "null pointer argument");
  if (flags & ~FGMM_STEP_PREPARED) return fail(FGMM_ERR_INVALID, "unknown flags");
  const bool prepared = (flags & FGMM_STEP_PREPARED) != 0;
  if (prepared && (!points || resolve_family(N, d, K) != FGMM_FAMILY_TC))
    return fail(FGMM_ERR_INVALID, "FGMM_STEP_PREPARED needs the tensor-core family and prepared points");
  fgmm::UpdateOut up{};
  up.n_total = (double)N;
  up.mu = new_mu;
  up.var = new_var;
  up.log_pi = new_log_pi;
  up.floors = true;
  return em_stats_impl(X, points, N, d, mu, var, log_pi, K, stats, log_normalizer, workspace,
                       workspace_bytes, stream, &up, prepared);
}

int fgmm_em_update(const double *stats, double n_total, int32_t K, int32_t d, float *new_mu,
                   float *new_var, float *new_log_pi, void *stream) {
  if (K < 1 || d < 1) return fail(FGMM_ERR_INVALID, "K and d must be >= 1");
  if (!stats || !new_mu || !new_var || !new_log_pi) return fail(FGMM_ERR_INVALID, "null pointer");
  if (!(n_total > 0)) return fail(FGMM_ERR_INVALID, "n_total must be > 0");
  return em_update(stats, n_total, K, d, new_mu, new_var, new_log_pi, (cudaStream_t)stream);
}

int fgmm_em_update_ex(const double *stats, double n_total, int32_t K, int32_t d, int32_t flags,
                      float *new_mu, float *new_var, float *new_log_pi, void *stream) {
  if (K < 1 || d < 1) return fail(FGMM_ERR_INVALID, "K and d must be >= 1");
  if (!stats || !new_mu || !new_var || !new_log_pi) return fail(FGMM_ERR_INVALID, "null pointer");
  if (!(n_total > 0)) return fail(FGMM_ERR_INVALID, "n_total must be > 0");
  if (flags & ~FGMM_UPDATE_NO_FLOORS) return fail(FGMM_ERR_INVALID, "unknown flags");
  return em_update(stats, n_total, K, d, new_mu, new_var, new_log_pi, (cudaStream_t)stream,
                   (flags & FGMM_UPDATE_NO_FLOORS) == 0);
}

size_t fgmm_em_fused_workspace_bytes(int64_t N, int32_t d, int32_t K) {
  int fam = resolve_family(N, d, K);
  if (fam < 0) return 0;
  size_t b = align_up(fgmm_em_stats_workspace_bytes(N, d, K), 256);
  if (fam == FGMM_FAMILY_TC) b += align_up(tc_points_bytes(N, d), 256);
  b += align_up((size_t)fgmm_stats_len(K, d) * sizeof(double), 256);
  return b;
}

int fgmm_em_fused(const float *X, int64_t N, int32_t d, const float *mu, const float *var,
                  const float *log_pi, int32_t K, float *new_mu, float *new_var,
                  float *new_log_pi, float *log_normalizer, void *workspace,
                  size_t workspace_bytes, void *stream) {
  int rc = check_shape(N, d, K);
  if (rc) return rc;
  if (!workspace) return fail(FGMM_ERR_INVALID, "null workspace");
  const size_t need = fgmm_em_fused_workspace_bytes(N, d, K);
  if (workspace_bytes < need) return fail(FGMM_ERR_WORKSPACE, "workspace too small");
  // stats live at the end; the stats workspace (+ in-place points) at the front
  const size_t stats_off = need - align_up((size_t)fgmm_stats_len(K, d) * sizeof(double), 256);
  double *stats = reinterpret_cast<double *>(static_cast<char *>(workspace) + stats_off);
  if (!new_mu || !new_var || !new_log_pi) return fail(FGMM_ERR_INVALID, "null pointer");
  const fgmm::UpdateOut up{(double)N, new_mu, new_var, new_log_pi, true};
  return em_stats_impl(X, nullptr, N, d, mu, var, log_pi, K, stats, log_normalizer, workspace,
                       stats_off, stream, &up);
}

size_t fgmm_e_step_workspace_bytes(int64_t N, int32_t d, int32_t K) {
  if (N < 1 || K < 1 || d < 1 || d > 256) return 0;
  return estep_workspace_bytes(N, d, K);
}

int fgmm_e_step(const float *X, int64_t N, int32_t d, const float *mu, const float *var,
                const float *log_pi, int32_t K, float *gamma, float *log_normalizer,
                void *workspace, size_t workspace_bytes, void *stream) {
  int rc = check_shape(N, d, K);
  if (rc) return rc;
  if (!X || !mu || !var || !log_pi || !gamma || !log_normalizer || !workspace)
    return fail(FGMM_ERR_INVALID, "null pointer argument");
  if (!aligned(workspace, 256)) return fail(FGMM_ERR_INVALID, "workspace must be 256-byte aligned");
  if (workspace_bytes < estep_workspace_bytes(N, d, K))
    return fail(FGMM_ERR_WORKSPACE, "workspace too small");
  return estep(X, N, d, mu, var, log_pi, K, gamma, log_normalizer, workspace, (cudaStream_t)stream);
}

size_t fgmm_m_step_workspace_bytes(int64_t N, int32_t d, int32_t K) {
  if (N < 1 || K < 1 || d < 1 || d > 256) return 0;
  return align_up(mstep_workspace_bytes(N, d, K), 256) +
         align_up((size_t)fgmm_stats_len(K, d) * sizeof(double), 256);
}

int fgmm_m_step(const float *X, int64_t N, int32_t d, const float *gamma, int32_t K,
                float *new_mu, float *new_var, float *new_log_pi, void *workspace,
                size_t workspace_bytes, void *stream) {
  int rc = check_shape(N, d, K);
  if (rc) return rc;
  if (!X || !gamma || !new_mu || !new_var || !new_log_pi || !workspace)
    return fail(FGMM_ERR_INVALID, "null pointer argument");
  if (!aligned(workspace, 256)) return fail(FGMM_ERR_INVALID, "workspace must be 256-byte aligned");
  const size_t need = fgmm_m_step_workspace_bytes(N, d, K);
  if (workspace_bytes < need) return fail(FGMM_ERR_WORKSPACE, "workspace too small");
  const size_t stats_off = align_up(mstep_workspace_bytes(N, d, K), 256);
  double *stats = reinterpret_cast<double *>(static_cast<char *>(workspace) + stats_off);
  cudaStream_t st = (cudaStream_t)stream;
  rc = mstep_stats(X, N, d, gamma, K, stats, workspace, st);
  if (rc) return rc;
  return em_update(stats, (double)N, K, d, new_mu, new_var, new_log_pi, st, /*floors=*/false);
}

int fgmm_device_error(int reset) { return tc_device_error(reset != 0); }

int fgmm_em_stats_launches(int64_t N, int32_t d, int32_t K) {
  const int fam = resolve_family(N, d, K);
  if (fam == FGMM_FAMILY_SIMT) return simt_launches();
  if (fam == FGMM_FAMILY_LOWK) return lowk_launches();
  if (fam == FGMM_FAMILY_TC) return tc_launches(N, d, K);
  return 0;
}

int fgmm_em_stats_profiled(const float *X, const void *points, int64_t N, int32_t d,
                           const float *mu, const float *var, const float *log_pi, int32_t K,
                           double *stats, float *log_normalizer, void *workspace,
                           size_t workspace_bytes, void *stream, float *launch_ms,
                           const char **names, int32_t n) {
  PhaseTimer t;
  for (int i = 0; i <= PhaseTimer::kMax; ++i) FGMM_CUDA_TRY(cudaEventCreate(&t.ev[i]));
  cudaStream_t st = (cudaStream_t)stream;
  cudaEventRecord(t.ev[0], st);
  phase_timer() = &t;
  int rc = fgmm_em_stats(X, points, N, d, mu, var, log_pi, K, stats, log_normalizer, workspace,
                         workspace_bytes, stream);
  phase_timer() = nullptr;
  cudaError_t e = cudaStreamSynchronize(st);
  if (rc == FGMM_OK && e != cudaSuccess) rc = cuda_fail(e, "cudaStreamSynchronize");
  if (rc == FGMM_OK) {
    for (int i = 0; i < t.n && i < n; ++i) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, t.ev[i], t.ev[i + 1]);
      if (launch_ms) launch_ms[i] = ms;
      if (names) names[i] = t.name[i];
    }
  }
  for (int i = 0; i <= PhaseTimer::kMax; ++i) cudaEventDestroy(t.ev[i]);
  return rc;
}

}  // extern "C"
