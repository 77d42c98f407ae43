// E-step with materialised responsibilities: gamma[N][K] and the log-normalizer, for the
// reference's `standard_e_step` / `flash_e_step` ops (flash_gmm/csrc/binding.cpp:35-60;
// CUDA kernels flash_gmm/csrc/flash_gmm_cuda.cu:328-374, CPU flash_gmm_cpu.cpp:51-168).
//
// The log-likelihood is evaluated in the reference's direct form
//   L[n,k] = log_pi_k - 1/2 (d log 2pi + sum_j log var_kj + sum_j (x_nj - mu_kj)^2 / var_kj)
// with (x - mu) / sqrt(var) = x * var^-1/2 - mu * var^-1/2 formed by one FMA, on tiles of
// 64 points x 32 components (dimensions staged through shared memory in 32-wide chunks),
// written straight into the gamma buffer together with a per-(point, tile) (max, sum of
// exp) pair.  A second kernel merges the tiles' pairs into the log-normalizer and turns
// L into gamma = exp(L - ln) in place.  Both kernels are fp32 CUDA-core code: the E-step
// output is N x K, so it is bound by writing that matrix, not by the contraction.
#include "fgmm_common.cuh"

namespace fgmm {
namespace {

constexpr int kEPts = 64;    // points per tile (8 per warp)
constexpr int kEComps = 32;  // components per tile (one per lane)
constexpr int kEDim = 32;    // dimensions per shared-memory chunk

__global__ void __launch_bounds__(256)
estep_ll_kernel(const float *__restrict__ X, int64_t N, int d, const float *__restrict__ sc,
                const float *__restrict__ ms, const float *__restrict__ lc, int K,
                float *__restrict__ L, float *__restrict__ part_m, float *__restrict__ part_s,
                int T) {
  __shared__ float xs[kEPts][kEDim + 1];
  __shared__ float ss[kEDim][kEComps], mm[kEDim][kEComps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tk = blockIdx.y;  // component tiles in y (K / 32 <= 65535), point tiles in x
  const int k = tk * kEComps + lane;
  const int64_t n0 = (int64_t)blockIdx.x * kEPts;
  float acc[8];
#pragma unroll
  for (int p = 0; p < 8; ++p) acc[p] = 0.0f;
  for (int j0 = 0; j0 < d; j0 += kEDim) {
    for (int i = threadIdx.x; i < kEPts * kEDim; i += 256) {
      const int p = i / kEDim, j = i % kEDim;
      const int64_t n = n0 + p;
      xs[p][j] = (n < N && j0 + j < d) ? __ldg(X + n * d + j0 + j) : 0.0f;
    }
    for (int i = threadIdx.x; i < kEComps * kEDim; i += 256) {
      const int c = i / kEDim, j = i % kEDim;  // read along d, store transposed
      const int kk = tk * kEComps + c;
      const bool in = kk < K && j0 + j < d;
      ss[j][c] = in ? __ldg(sc + (int64_t)kk * d + j0 + j) : 0.0f;
      mm[j][c] = in ? __ldg(ms + (int64_t)kk * d + j0 + j) : 0.0f;
    }
    __syncthreads();
    const int jn = min(kEDim, d - j0);
    for (int j = 0; j < jn; ++j) {
      const float s = ss[j][lane], m = mm[j][lane];
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        const float w = fmaf(xs[warp * 8 + p][j], s, -m);
        acc[p] = fmaf(w, w, acc[p]);
      }
    }
    __syncthreads();
  }
  const float c = k < K ? __ldg(lc + k) : 0.0f;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const int64_t n = n0 + warp * 8 + p;
    const float l = k < K ? c - 0.5f * acc[p] : -INFINITY;
    if (n < N && k < K) L[n * K + k] = l;
    float mx = l;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float e = k < K ? expf(l - mx) : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    if (lane == 0 && n < N) {
      part_m[n * T + tk] = mx;
      part_s[n * T + tk] = e;
    }
  }
}

// One warp per point: merge the T tile pairs, write ln, turn L into gamma in place.
__global__ void __launch_bounds__(256)
estep_norm_kernel(int64_t N, int K, int T, const float *__restrict__ part_m,
                  const float *__restrict__ part_s, float *__restrict__ G,
                  float *__restrict__ ln_out) {
  const int lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (n >= N) return;
  float mx = -INFINITY;
  for (int t = lane; t < T; t += 32) mx = fmaxf(mx, part_m[n * T + t]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = 0.0f;
  for (int t = lane; t < T; t += 32) s += part_s[n * T + t] * expf(part_m[n * T + t] - mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float ln = mx + logf(s);
  if (lane == 0) ln_out[n] = ln;
  float *g = G + n * K;
  for (int k = lane; k < K; k += 32) g[k] = expf(g[k] - ln);
}

struct EstepWs {
  float *sc, *ms, *lc, *part_m, *part_s;
  int T;
  size_t bytes;
};

EstepWs estep_layout(void *ws, int64_t N, int d, int K) {
  EstepWs w{};
  Carve c(ws);
  w.T = (int)cdiv(K, kEComps);
  w.sc = c.take<float>((size_t)K * d);
  w.ms = c.take<float>((size_t)K * d);
  w.lc = c.take<float>(K);
  w.part_m = c.take<float>((size_t)N * w.T);
  w.part_s = c.take<float>((size_t)N * w.T);
  w.bytes = c.bytes();
  return w;
}

}  // namespace

size_t estep_workspace_bytes(int64_t N, int d, int K) { return estep_layout(nullptr, N, d, K).bytes; }

int estep(const float *X, int64_t N, int d, const float *mu, const float *var, const float *log_pi,
          int K, float *gamma, float *log_norm, void *ws, cudaStream_t st) {
  const EstepWs w = estep_layout(ws, N, d, K);
  int rc = prep_direct_params(mu, var, log_pi, K, d, w.sc, w.ms, w.lc, st);
  if (rc) return rc;
  if (cdiv(N, kEPts) > 0x7fffffff || w.T > 65535)
    return fail(FGMM_ERR_UNSUPPORTED, "E-step: N or K beyond the launch grid");
  dim3 grid((unsigned)cdiv(N, kEPts), w.T);
  estep_ll_kernel<<<grid, 256, 0, st>>>(X, N, d, w.sc, w.ms, w.lc, K, gamma, w.part_m, w.part_s, w.T);
  FGMM_LAUNCH_CHECK("estep_ll_kernel");
  estep_norm_kernel<<<(unsigned)cdiv(N, 8), 256, 0, st>>>(N, K, w.T, w.part_m, w.part_s, gamma, log_norm);
  FGMM_LAUNCH_CHECK("estep_norm_kernel");
  return FGMM_OK;
}

}  // namespace fgmm
